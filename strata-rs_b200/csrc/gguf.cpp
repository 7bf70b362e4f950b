// gguf.cpp — the GGUF reader behind include/strata_gguf.h and the bulk ingest
// of a model's tensors.
//
// A restatement of strata-gguf's reader (crates/strata-gguf/src/reader.rs)
// with the same bounds checks, limits and errors, so a model that one of them
// opens the other opens too, and each failure carries the same error:
//   layout (v3, little endian): magic "GGUF" | version u32 | tensor_count u64 |
//   kv_count u64 | kv_count x (key string, type u32, value) | tensor_count x
//   (name string, n_dims u32, dims u64 x n_dims, type u32, offset u64) |
//   padding to the alignment | data (tensor offsets count from here).
// Each shard is mapped read-only; a tensor's payload is a pointer into the
// mapping, which strata_cuda_gguf_ingest streams to HBM through the upload's
// pinned chunks (the host threads that fill a chunk take the page faults).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cinttypes>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/strata_gguf.h"
#include "host.h"

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" read as a little-endian u32
constexpr uint32_t kVersion = 3;
constexpr uint64_t kMaxArrayLen = uint64_t(1) << 24;  // plausibility limit on array counts
constexpr uint64_t kMaxString = 65535;
constexpr uint64_t kKeepAllItems = uint64_t(1) << 20;  // arrays up to this long are read through
constexpr uint64_t kItemsKept = 64;                    // longer ones: this many items are read
constexpr int kMaxDepth = 2;                           // array nesting the reader accepts

// A failure: a status code of strata_gguf.h and strata_gguf::Error's text.
struct GgufError {
    int code = STRATA_OK;
    std::string msg;
};

GgufError make_error(int code, const char* fmt, ...) {
    char buf[768];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return {code, buf};
}

GgufError truncated(uint64_t expected, uint64_t found) {
    return make_error(STRATA_ERR_TRUNCATED, "truncated GGUF file: expected %" PRIu64 " more bytes, found %" PRIu64,
                      expected, found);
}

GgufError io_error(const std::string& path, const std::string& why) {
    return make_error(STRATA_ERR_IO, "cannot open GGUF file '%s': %s", path.c_str(), why.c_str());
}

std::string os_error(int e) { return std::string(strerror(e)) + " (os error " + std::to_string(e) + ")"; }

// Elements per block and bytes per block of every Strata ggml type id
// (crates/strata-gguf/src/quant.rs:125-170); false for an unknown id.
bool type_geometry(uint32_t id, uint64_t* bs, uint64_t* ts) {
    struct G {
        uint32_t id, bs, ts;
    };
    static const G table[] = {
        {0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {6, 32, 22},   {7, 32, 24},   {8, 32, 34},
        {9, 32, 36},   {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176}, {14, 256, 210},
        {16, 256, 66}, {17, 256, 74}, {18, 256, 98},  {20, 32, 18},   {21, 256, 110}, {22, 256, 82},
        {23, 256, 136}, {24, 1, 1},   {29, 256, 56},  {30, 1, 2},     {39, 32, 17},   {40, 64, 36},
        {41, 128, 18}, {42, 64, 18},
    };
    for (const G& g : table)
        if (g.id == id) {
            *bs = g.bs;
            *ts = g.ts;
            return true;
        }
    return false;
}

// Strict UTF-8, as Rust's str::from_utf8: no overlong forms, no surrogates,
// nothing above U+10FFFF.
bool valid_utf8(const uint8_t* p, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = p[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        int extra;
        uint8_t lo = 0x80, hi = 0xBF;
        if (c >= 0xC2 && c <= 0xDF) {
            extra = 1;
        } else if (c >= 0xE0 && c <= 0xEF) {
            extra = 2;
            if (c == 0xE0) lo = 0xA0;
            if (c == 0xED) hi = 0x9F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            extra = 3;
            if (c == 0xF0) lo = 0x90;
            if (c == 0xF4) hi = 0x8F;
        } else {
            return false;
        }
        if (n - i <= (size_t)extra) return false;
        if (p[i + 1] < lo || p[i + 1] > hi) return false;
        for (int k = 2; k <= extra; ++k)
            if (p[i + k] < 0x80 || p[i + k] > 0xBF) return false;
        i += extra + 1;
    }
    return true;
}

struct Value {
    uint32_t ty = 0;
    int64_t i = 0;
    uint64_t u = 0;
    double f = 0;
    std::string s;
    uint32_t elem = STRATA_GGUF_U32;
    uint64_t count = 0;
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> shape;
    uint32_t ty = 0;
    uint64_t offset = 0;
};

// A bounds-checked little-endian reader over the mapped file; every read
// past the end is Truncated with the bytes still left.
struct Cursor {
    const uint8_t* p;
    uint64_t n;
    uint64_t pos = 0;

    bool need(uint64_t k, GgufError* e) const {
        if (k > n - pos) {
            *e = truncated(k, n - pos);
            return false;
        }
        return true;
    }
    template <typename T>
    bool get(T* v, GgufError* e) {
        if (!need(sizeof(T), e)) return false;
        memcpy(v, p + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool string(std::string* s, GgufError* e) {
        uint64_t len;
        if (!get(&len, e)) return false;
        if (len > kMaxString) {
            *e = make_error(STRATA_ERR_BAD_KEY_LENGTH, "invalid metadata key length %" PRIu64 " (max 65535)", len);
            return false;
        }
        if (!need(len, e)) return false;
        if (!valid_utf8(p + pos, len)) {
            *e = make_error(STRATA_ERR_STRING_NOT_UTF8, "string is not valid UTF-8");
            return false;
        }
        s->assign(reinterpret_cast<const char*>(p + pos), len);
        pos += len;
        return true;
    }
};

bool value_type(uint32_t id, GgufError* e) {
    if (id <= STRATA_GGUF_F64) return true;
    *e = make_error(STRATA_ERR_BAD_VALUE_TYPE, "invalid metadata value type %u", id);
    return false;
}

// One metadata value of type `ty` (Cursor::value, reader.rs:123-174).
// Arrays keep their element type and count; their items are read through
// (all of them up to 2^20 items, else the first 64, as the reference does)
// and not kept.
bool read_value(Cursor& c, uint32_t ty, int depth, Value* v, GgufError* e) {
    if (depth > kMaxDepth) {
        *e = make_error(STRATA_ERR_BAD_VALUE_TYPE, "invalid metadata value type %u", (unsigned)STRATA_GGUF_ARRAY);
        return false;
    }
    v->ty = ty;
    switch (ty) {
        case STRATA_GGUF_U8: { uint8_t x; if (!c.get(&x, e)) return false; v->i = x; return true; }
        case STRATA_GGUF_I8: { int8_t x; if (!c.get(&x, e)) return false; v->i = x; return true; }
        case STRATA_GGUF_U16: { uint16_t x; if (!c.get(&x, e)) return false; v->i = x; return true; }
        case STRATA_GGUF_I16: { int16_t x; if (!c.get(&x, e)) return false; v->i = x; return true; }
        case STRATA_GGUF_U32: { uint32_t x; if (!c.get(&x, e)) return false; v->i = x; return true; }
        case STRATA_GGUF_I32: { int32_t x; if (!c.get(&x, e)) return false; v->i = x; return true; }
        case STRATA_GGUF_F32: { float x; if (!c.get(&x, e)) return false; v->f = x; return true; }
        case STRATA_GGUF_BOOL: { uint8_t x; if (!c.get(&x, e)) return false; v->i = x != 0; return true; }
        case STRATA_GGUF_STRING: return c.string(&v->s, e);
        case STRATA_GGUF_U64: return c.get(&v->u, e);
        case STRATA_GGUF_I64: return c.get(&v->i, e);
        case STRATA_GGUF_F64: return c.get(&v->f, e);
        case STRATA_GGUF_ARRAY: {
            uint32_t elem;
            if (!c.get(&elem, e) || !value_type(elem, e)) return false;
            uint64_t count;
            if (!c.get(&count, e)) return false;
            if (count > kMaxArrayLen) {
                *e = make_error(STRATA_ERR_BAD_VALUE_TYPE, "invalid metadata value type %u",
                                (unsigned)STRATA_GGUF_ARRAY);
                return false;
            }
            v->elem = elem;
            v->count = count;
            const uint64_t read = count <= kKeepAllItems ? count : kItemsKept;
            Value item;
            for (uint64_t k = 0; k < read; ++k)
                if (!read_value(c, elem, depth + 1, &item, e)) return false;
            return true;
        }
        default: return value_type(ty, e);
    }
}

struct Shard {
    std::string path;
    const uint8_t* base = nullptr;  // the read-only mapping (nullptr for an empty file)
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_start = 0;
    std::vector<TensorInfo> tensors;
    std::unordered_map<std::string, Value> meta;

    Shard() = default;
    Shard(const Shard&) = delete;
    Shard& operator=(const Shard&) = delete;
    ~Shard() {
        if (base) munmap(const_cast<uint8_t*>(base), size);
    }
};

// GgufFile::open + parse (reader.rs:231-352).
bool open_shard(const std::string& path, Shard* sh, GgufError* e) {
    sh->path = path;
    // non-blocking open: a FIFO or device node is refused below instead of blocking here
    const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC | O_NONBLOCK);
    if (fd < 0) {
        *e = io_error(path, os_error(errno));
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        const int err = errno;
        close(fd);
        *e = io_error(path, os_error(err));
        return false;
    }
    if (!S_ISREG(st.st_mode)) {
        close(fd);
        *e = io_error(path, S_ISDIR(st.st_mode) ? "is a directory" : "not a regular file");
        return false;
    }
    sh->size = (uint64_t)st.st_size;
    if (sh->size > 0) {
        void* m = mmap(nullptr, sh->size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) {
            const int err = errno;
            close(fd);
            *e = io_error(path, os_error(err));
            return false;
        }
        sh->base = static_cast<const uint8_t*>(m);
        madvise(m, sh->size, MADV_SEQUENTIAL);
    }
    close(fd);

    Cursor c{sh->base, sh->size};
    uint32_t magic;
    if (!c.get(&magic, e)) return false;
    if (magic != kMagic) {
        *e = make_error(STRATA_ERR_BAD_MAGIC, "not a GGUF file (bad magic %#x)", magic);
        return false;
    }
    if (!c.get(&sh->version, e)) return false;
    if (sh->version != kVersion) {
        *e = make_error(STRATA_ERR_UNSUPPORTED_VERSION, "unsupported GGUF version %u (expected 2 or 3)", sh->version);
        return false;
    }
    uint64_t n_tensors, n_kv;
    if (!c.get(&n_tensors, e) || !c.get(&n_kv, e)) return false;
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key;
        uint32_t ty;
        Value v;
        if (!c.string(&key, e) || !c.get(&ty, e) || !value_type(ty, e) || !read_value(c, ty, 0, &v, e)) return false;
        sh->meta[key] = std::move(v);
    }
    std::unordered_map<std::string, size_t> names;
    for (uint64_t k = 0; k < n_tensors; ++k) {
        TensorInfo t;
        if (!c.string(&t.name, e)) return false;
        if (!names.emplace(t.name, sh->tensors.size()).second) {
            *e = make_error(STRATA_ERR_TENSOR_NOT_FOUND, "tensor '%s' is missing from the file", t.name.c_str());
            return false;
        }
        uint32_t nd;
        if (!c.get(&nd, e)) return false;
        if (nd == 0 || nd > 4) {
            *e = make_error(STRATA_ERR_WRONG_TENSOR_DIMS, "tensor '%s' has %u dimensions, expected 4", t.name.c_str(),
                            nd);
            return false;
        }
        t.shape.resize(nd);
        for (uint32_t d = 0; d < nd; ++d)
            if (!c.get(&t.shape[d], e)) return false;
        if (!c.get(&t.ty, e) || !c.get(&t.offset, e)) return false;
        sh->tensors.push_back(std::move(t));
    }
    // general.alignment counts when it is a positive integer held in the
    // signed payload (MetaValue::as_int): the 8- to 32-bit types, bool, i64.
    // A u64 value keeps its payload elsewhere and so leaves the default.
    auto it = sh->meta.find("general.alignment");
    if (it != sh->meta.end()) {
        const uint32_t t = it->second.ty;
        const bool is_int = t != STRATA_GGUF_F32 && t != STRATA_GGUF_F64 && t != STRATA_GGUF_STRING &&
                            t != STRATA_GGUF_ARRAY;
        if (is_int && it->second.i > 0) sh->alignment = (uint64_t)it->second.i;
    }
    const uint64_t data_start = (c.pos + sh->alignment - 1) / sh->alignment * sh->alignment;
    if (data_start > sh->size) {
        if (!sh->tensors.empty()) {
            *e = truncated(data_start, sh->size);
            return false;
        }
        sh->data_start = sh->size;  // a metadata-only shard may end before the aligned data start
    } else {
        sh->data_start = data_start;
    }
    return true;
}

// split_paths (reader.rs:527-572): the shards of `<stem>-NNNNN-of-MMMMM.gguf`
// in order, or the path itself when it does not have that shape.
bool split_paths(const std::string& s, std::vector<std::string>* out, GgufError* e) {
    out->clear();
    const size_t at = s.rfind("-of-");
    const bool shaped = at != std::string::npos && at >= 6 && s[at - 6] == '-' && s.size() == at + 14 &&
                        s.compare(at + 9, 5, ".gguf") == 0;
    uint64_t no = 0, n = 0;
    bool digits = shaped;
    for (int i = 0; digits && i < 5; ++i) {
        const char a = s[at - 5 + i], b = s[at + 4 + i];
        if (a < '0' || a > '9' || b < '0' || b > '9') digits = false;
        no = no * 10 + (uint64_t)(a - '0');
        n = n * 10 + (uint64_t)(b - '0');
    }
    if (!digits || n < 1 || no < 1 || no > n) {
        out->push_back(s);
        return true;
    }
    for (uint64_t i = 1; i <= n; ++i) {
        char num[8];
        snprintf(num, sizeof(num), "%05" PRIu64, i);
        std::string p = s;
        p.replace(at - 5, 5, num);
        struct stat st;
        if (stat(p.c_str(), &st) != 0) {
            char why[96];
            snprintf(why, sizeof(why), "missing model shard %" PRIu64 " of %" PRIu64 " (is the download complete?)", i,
                     n);
            *e = io_error(p, why);
            return false;
        }
        out->push_back(std::move(p));
    }
    return true;
}

void put_error(const GgufError& ge, char* err, size_t err_len) {
    if (err && err_len) snprintf(err, err_len, "%s", ge.msg.c_str());
}

}  // namespace

struct strata_gguf {
    std::vector<Shard*> shards;
    std::vector<std::pair<int, size_t>> order;      // (shard, tensor) in shard then directory order
    std::unordered_map<std::string, int64_t> index;  // name -> position in `order`

    ~strata_gguf() {
        for (Shard* s : shards) delete s;
    }
    const TensorInfo& tensor(int64_t i) const { return shards[order[i].first]->tensors[order[i].second]; }
};

namespace {

// GgufFile::tensor_payload_bytes + tensor_data (reader.rs:399-445). The byte
// count n_blocks * type_size is checked for overflow as well (Truncated).
bool tensor_payload(const Shard& sh, const TensorInfo& t, const uint8_t** data, uint64_t* nbytes, GgufError* e) {
    if (t.shape.empty()) {
        *e = make_error(STRATA_ERR_WRONG_TENSOR_DIMS, "tensor '%s' has 0 dimensions, expected 4", t.name.c_str());
        return false;
    }
    uint64_t bs, ts;
    if (!type_geometry(t.ty, &bs, &ts)) {
        *e = make_error(STRATA_ERR_UNSUPPORTED_QUANT, "unsupported quantization type \"type id %u\"", t.ty);
        return false;
    }
    uint64_t elems = 1;
    for (uint64_t d : t.shape) {
        if (d == 0 || elems > UINT64_MAX / d) {
            *e = truncated(t.offset, 0);
            return false;
        }
        elems *= d;
    }
    const uint64_t blocks = elems / bs;
    if (blocks > UINT64_MAX / ts) {
        *e = truncated(t.offset, 0);
        return false;
    }
    const uint64_t bytes = blocks * ts;
    if (t.offset > UINT64_MAX - sh.data_start) {
        *e = truncated(t.offset, 0);
        return false;
    }
    const uint64_t start = sh.data_start + t.offset;
    if (bytes > UINT64_MAX - start) {
        *e = truncated(bytes, 0);
        return false;
    }
    if (start + bytes > sh.size) {
        *e = truncated(bytes, sh.size > start ? sh.size - start : 0);
        return false;
    }
    *data = sh.base ? sh.base + start : nullptr;
    *nbytes = bytes;
    return true;
}

// The upload item for rows [first, first + count) of a 1-D / 2-D tensor or
// experts [first, first + count) of a 3-D one, viewed as WeightStore views it
// (weights.rs:122-152): 1-D one row of dims[0]; 2-D [cols, rows]; 3-D
// [cols, rows, n_expert]. count < 0 means to the end.
bool tensor_view(const strata_gguf& g, int64_t index, int64_t first, int64_t count, strata_upload* u,
                 GgufError* e) {
    const Shard& sh = *g.shards[g.order[index].first];
    const TensorInfo& t = g.tensor(index);
    const uint8_t* data;
    uint64_t nbytes;
    if (!tensor_payload(sh, t, &data, &nbytes, e)) return false;
    for (uint64_t d : t.shape)
        if (d > (uint64_t)INT64_MAX) {
            *e = make_error(STRATA_ERR_INVALID, "tensor '%s' has a dimension beyond int64", t.name.c_str());
            return false;
        }
    const int nd = (int)t.shape.size();
    if (nd > 3) {
        *e = make_error(STRATA_ERR_INVALID, "tensor '%s' has %d dimensions; a weight view has 1 to 3", t.name.c_str(),
                        nd);
        return false;
    }
    const int64_t cols = (int64_t)t.shape[0];
    const int64_t rows = nd == 1 ? 1 : (int64_t)t.shape[1];
    const int64_t outer = nd == 3 ? (int64_t)t.shape[2] : rows;  // what [first, first + count) counts
    const char* what = nd == 3 ? "experts" : "rows";
    if (first < 0 || first > outer) {
        *e = make_error(STRATA_ERR_INVALID, "first %s %lld is outside tensor '%s' (%lld %s)", what, (long long)first,
                        t.name.c_str(), (long long)outer, what);
        return false;
    }
    if (count < 0) count = outer - first;
    if (count > outer - first) {
        *e = make_error(STRATA_ERR_INVALID, "%lld %s from %lld run past the end of tensor '%s' (%lld %s)",
                        (long long)count, what, (long long)first, t.name.c_str(), (long long)outer, what);
        return false;
    }
    uint64_t bs = 1, ts = 0;
    type_geometry(t.ty, &bs, &ts);  // known: the payload was found
    const uint64_t row_bytes = ((uint64_t)cols + bs - 1) / bs * ts;
    const uint64_t unit = nd == 3 ? row_bytes * (uint64_t)rows : row_bytes;  // bytes per counted item
    if (unit && (uint64_t)outer > nbytes / unit) {
        *e = truncated(unit * (uint64_t)outer, nbytes);  // rows that are not whole blocks
        return false;
    }
    u->bytes = data ? data + unit * (uint64_t)first : nullptr;
    u->len = (size_t)(unit * (uint64_t)count);
    u->quant = t.ty;
    u->cols = cols;
    u->n_expert = nd == 3 ? count : 0;
    u->rows = nd == 3 ? rows : count;
    return true;
}

}  // namespace

extern "C" {

int strata_cuda_gguf_split_paths(const char* any_shard, char* buf, size_t buf_len, size_t* needed, char* err,
                                 size_t err_len) {
    if (!any_shard) return STRATA_ERR_INVALID;
    std::vector<std::string> paths;
    GgufError e;
    if (!split_paths(any_shard, &paths, &e)) {
        put_error(e, err, err_len);
        return e.code;
    }
    std::string all;
    for (const std::string& p : paths) all += p + "\n";
    if (needed) *needed = all.size() + 1;
    if (!buf || buf_len < all.size() + 1) return STRATA_ERR_INVALID;
    memcpy(buf, all.c_str(), all.size() + 1);
    return STRATA_OK;
}

int strata_cuda_gguf_open(const char* any_shard, strata_gguf** out, char* err, size_t err_len) {
    if (!any_shard || !out) return STRATA_ERR_INVALID;
    *out = nullptr;
    std::vector<std::string> paths;
    GgufError e;
    if (!split_paths(any_shard, &paths, &e)) {
        put_error(e, err, err_len);
        return e.code;
    }
    strata_gguf* g = new strata_gguf();
    for (const std::string& p : paths) {
        Shard* sh = new Shard();
        g->shards.push_back(sh);
        if (!open_shard(p, sh, &e)) {
            delete g;
            put_error(e, err, err_len);
            return e.code;
        }
    }
    for (size_t si = 0; si < g->shards.size(); ++si)
        for (size_t ti = 0; ti < g->shards[si]->tensors.size(); ++ti) {
            const std::string& name = g->shards[si]->tensors[ti].name;
            if (!g->index.emplace(name, (int64_t)g->order.size()).second) {
                e = make_error(STRATA_ERR_TENSOR_NOT_FOUND, "tensor '%s' is missing from the file", name.c_str());
                delete g;
                put_error(e, err, err_len);
                return e.code;
            }
            g->order.emplace_back((int)si, ti);
        }
    *out = g;
    return STRATA_OK;
}

void strata_cuda_gguf_close(strata_gguf* g) { delete g; }

int strata_cuda_gguf_n_shards(const strata_gguf* g) { return g ? (int)g->shards.size() : 0; }

int strata_cuda_gguf_shard(const strata_gguf* g, int shard, strata_gguf_shard* out) {
    if (!g || !out || shard < 0 || shard >= (int)g->shards.size()) return STRATA_ERR_INVALID;
    const Shard& s = *g->shards[shard];
    out->path = s.path.c_str();
    out->version = s.version;
    out->alignment = s.alignment;
    out->data_start = s.data_start;
    out->file_size = s.size;
    out->n_tensors = (int64_t)s.tensors.size();
    out->n_metadata = (int64_t)s.meta.size();
    return STRATA_OK;
}

int64_t strata_cuda_gguf_tensor_count(const strata_gguf* g) { return g ? (int64_t)g->order.size() : 0; }

int strata_cuda_gguf_tensor(const strata_gguf* g, int64_t index, strata_gguf_tensor* out) {
    if (!g || !out || index < 0 || index >= (int64_t)g->order.size()) return STRATA_ERR_INVALID;
    const TensorInfo& t = g->tensor(index);
    out->name = t.name.c_str();
    out->name_len = t.name.size();
    out->type = t.ty;
    out->n_dims = (int32_t)t.shape.size();
    for (int d = 0; d < 4; ++d) out->dims[d] = d < (int)t.shape.size() ? t.shape[d] : 0;
    out->offset = t.offset;
    out->shard = g->order[index].first;
    return STRATA_OK;
}

int strata_cuda_gguf_find(const strata_gguf* g, const char* name, int64_t* index) {
    if (!g || !name || !index) return STRATA_ERR_INVALID;
    auto it = g->index.find(name);
    *index = it == g->index.end() ? -1 : it->second;
    return it == g->index.end() ? (int)STRATA_ERR_TENSOR_NOT_FOUND : (int)STRATA_OK;
}

int strata_cuda_gguf_tensor_data(const strata_gguf* g, int64_t index, const uint8_t** data, uint64_t* nbytes,
                                 char* err, size_t err_len) {
    if (!g || !data || !nbytes || index < 0 || index >= (int64_t)g->order.size()) return STRATA_ERR_INVALID;
    *data = nullptr;
    *nbytes = 0;
    GgufError e;
    if (!tensor_payload(*g->shards[g->order[index].first], g->tensor(index), data, nbytes, &e)) {
        put_error(e, err, err_len);
        return e.code;
    }
    return STRATA_OK;
}

int strata_cuda_gguf_meta(const strata_gguf* g, const char* key, strata_gguf_value* out) {
    if (!g || !key || !out || g->shards.empty()) return STRATA_ERR_INVALID;
    const auto& meta = g->shards[0]->meta;
    auto it = meta.find(key);
    if (it == meta.end()) return STRATA_ERR_INVALID;
    const Value& v = it->second;
    out->type = v.ty;
    out->i = v.i;
    out->u = v.u;
    out->f = v.f;
    out->str = v.s.c_str();
    out->str_len = v.s.size();
    out->elem = v.elem;
    out->count = v.count;
    return STRATA_OK;
}

int strata_cuda_gguf_view(const strata_gguf* g, int64_t index, int64_t first, int64_t count, strata_upload* out,
                          char* err, size_t err_len) {
    if (!g || !out || index < 0 || index >= (int64_t)g->order.size()) return STRATA_ERR_INVALID;
    GgufError e;
    if (!tensor_view(*g, index, first, count, out, &e)) {
        put_error(e, err, err_len);
        return e.code;
    }
    return STRATA_OK;
}

int strata_cuda_gguf_ingest(strata_ctx* ctx, const strata_gguf* g, const int64_t* tensors, int64_t n,
                            strata_weight** out) {
    if (!ctx || !g || n < 0 || (n > 0 && (!tensors || !out))) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::vector<strata_upload> items((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        const int64_t ix = tensors[i];
        GgufError e;
        if (ix < 0 || ix >= (int64_t)g->order.size())
            e = make_error(STRATA_ERR_INVALID, "tensor index %lld is out of range", (long long)ix);
        else if (tensor_view(*g, ix, 0, -1, &items[(size_t)i], &e) && !strata::quant_on_device(items[(size_t)i].quant))
            e = make_error(STRATA_ERR_UNSUPPORTED_QUANT, "tensor '%s': quant type id %u is not on the CUDA path",
                           g->tensor(ix).name.c_str(), items[(size_t)i].quant);
        else if (e.code == STRATA_OK)
            continue;
        for (int64_t k = 0; k < n; ++k) out[k] = nullptr;
        return strata::report(ctx, e.code, e.msg.c_str());
    }
    return strata_cuda_upload_many(ctx, items.data(), n, out);
}

int strata_cuda_gguf_moe_layer(strata_ctx* ctx, const strata_gguf* g, int64_t layer, int64_t top_k,
                               int64_t expert_begin, int64_t expert_end, int with_shared, strata_moe** out,
                               strata_weight** weights_out) {
    if (!ctx || !g || !out || !weights_out || layer < 0) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    *out = nullptr;
    for (int i = 0; i < 8; ++i) weights_out[i] = nullptr;
    // strata_moe_desc's order: router, gate/up/down experts, gate/up/down shared, shared gate input
    static const char* const kNames[8] = {"ffn_gate_inp",   "ffn_gate_exps",  "ffn_up_exps",
                                          "ffn_down_exps",  "ffn_gate_shexp", "ffn_up_shexp",
                                          "ffn_down_shexp", "ffn_gate_inp_shexp"};
    const int n_tensors = with_shared ? 8 : 4;
    const std::string prefix = "blk." + std::to_string(layer) + ".";
    int64_t index[8];
    for (int i = 0; i < n_tensors; ++i) {
        const std::string name = prefix + kNames[i] + ".weight";
        auto it = g->index.find(name);
        if (it == g->index.end())
            return strata::report(ctx, STRATA_ERR_TENSOR_NOT_FOUND,
                                  ("tensor '" + name + "' is missing from the model").c_str());
        index[i] = it->second;
    }
    // the expert count and range from gate_exps ([n_ff, n_embd, n_expert])
    const TensorInfo& ge = g->tensor(index[1]);
    if (ge.shape.size() != 3 || ge.shape[2] > (uint64_t)INT64_MAX)
        return strata::report(ctx, STRATA_ERR_WRONG_TENSOR_DIMS,
                              ("tensor '" + ge.name + "' is not a 3-D expert tensor").c_str());
    const int64_t n_expert = (int64_t)ge.shape[2];
    if (expert_end <= 0) expert_end = n_expert;
    if (expert_begin < 0 || expert_begin >= expert_end || expert_end > n_expert)
        return strata::report(ctx, STRATA_ERR_INVALID,
                              ("expert range [" + std::to_string(expert_begin) + ", " + std::to_string(expert_end) +
                               ") outside the " + std::to_string(n_expert) + " experts of '" + ge.name + "'")
                                  .c_str());
    strata_upload items[8];
    for (int i = 0; i < n_tensors; ++i) {
        const bool experts = i >= 1 && i <= 3;
        GgufError e;
        if (!tensor_view(*g, index[i], experts ? expert_begin : 0, experts ? expert_end - expert_begin : -1,
                         &items[i], &e))
            return strata::report(ctx, e.code, e.msg.c_str());
        if (experts != (items[i].n_expert > 0))
            return strata::report(ctx, STRATA_ERR_WRONG_TENSOR_DIMS,
                                  ("tensor '" + g->tensor(index[i]).name + "' has " +
                                   std::to_string(g->tensor(index[i]).shape.size()) + " dimensions")
                                      .c_str());
    }
    strata_weight* ws[8] = {};
    int rc = strata_cuda_upload_many(ctx, items, n_tensors, ws);
    if (rc) return rc;
    strata_moe_desc d{};
    d.router = ws[0];
    d.gate_exps = ws[1];
    d.up_exps = ws[2];
    d.down_exps = ws[3];
    d.gate_shexp = with_shared ? ws[4] : nullptr;
    d.up_shexp = with_shared ? ws[5] : nullptr;
    d.down_shexp = with_shared ? ws[6] : nullptr;
    d.gate_inp_shexp = with_shared ? ws[7] : nullptr;
    d.n_embd = items[0].cols;   // the router is [n_expert rows][n_embd]
    d.n_expert = n_expert;
    d.top_k = top_k;
    d.n_ff = items[1].cols;     // gate_exps' columns, as load_layer takes n_ff
    d.n_ff_shexp = with_shared ? items[4].rows : 0;
    d.expert_begin = expert_begin;
    d.expert_end = expert_end;
    d.with_shared = with_shared ? 1 : 0;
    rc = strata_cuda_moe_create(ctx, &d, out);
    if (rc) {
        for (int i = 0; i < n_tensors; ++i) strata_cuda_free_weight(ws[i]);
        return rc;
    }
    for (int i = 0; i < n_tensors; ++i) weights_out[i] = ws[i];
    return STRATA_OK;
}

}  // extern "C"
