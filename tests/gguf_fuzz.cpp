// Mutation fuzzing of the GGUF reader (strata-rs_b200/csrc/gguf.cpp), built
// as a host program with address and undefined-behaviour checks. Each seed
// file (a valid GGUF written by tests/gguf_writer.py) is mutated at random --
// bytes overwritten, runs of bytes zeroed or set to 0xFF, 64-bit fields set to
// extreme values, the file cut short or extended -- then opened; every tensor
// of a model that opens is asked for its payload and its views, and a few
// metadata keys are read. Any out-of-bounds access or undefined behaviour
// aborts the program; otherwise it prints "ok <opened> <refused>".
//
// Usage: gguf_fuzz <work-file> <iterations> <seed-file>...
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "../include/strata_gguf.h"

// The ingest and layer entry points link against these; the fuzzer never reaches them.
extern "C" int strata_cuda_upload_many(strata_ctx*, const strata_upload*, int64_t, strata_weight**) { return 1; }
extern "C" int strata_cuda_moe_create(strata_ctx*, const strata_moe_desc*, strata_moe**) { return 1; }
extern "C" int strata_cuda_free_weight(strata_weight*) { return 1; }
namespace strata {
int report(strata_ctx*, int code, const char*) { return code; }
bool quant_on_device(uint32_t) { return true; }
}  // namespace strata

static std::vector<uint8_t> read_file(const char* p) {
    std::vector<uint8_t> b;
    FILE* f = fopen(p, "rb");
    if (!f) return b;
    uint8_t buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof(buf), f)) > 0) b.insert(b.end(), buf, buf + n);
    fclose(f);
    return b;
}

static void write_file(const char* p, const std::vector<uint8_t>& b) {
    FILE* f = fopen(p, "wb");
    if (!f) {
        perror("fopen");
        exit(2);
    }
    if (!b.empty()) fwrite(b.data(), 1, b.size(), f);
    fclose(f);
}

static void mutate(std::vector<uint8_t>& b, std::mt19937_64& g) {
    const int n_mut = 1 + (int)(g() % 4);
    for (int m = 0; m < n_mut; ++m) {
        const size_t len = b.size();
        switch (g() % 7) {
            case 0:  // one byte
                if (len) b[g() % len] = (uint8_t)g();
                break;
            case 1:  // a run of zeros or 0xFF
                if (len) {
                    const size_t at = g() % len, k = 1 + g() % 16, v = (g() & 1) ? 0xFF : 0;
                    for (size_t i = at; i < len && i < at + k; ++i) b[i] = (uint8_t)v;
                }
                break;
            case 2:  // a 64-bit field set to an extreme value, at any offset
                if (len >= 8) {
                    static const uint64_t vals[] = {0, 1, 4, 5, 65535, 65536, (1ull << 24) + 1, (1ull << 20) + 1,
                                                    UINT32_MAX, (uint64_t)INT64_MAX, UINT64_MAX, UINT64_MAX - 15};
                    const uint64_t v = vals[g() % (sizeof(vals) / sizeof(vals[0]))];
                    memcpy(&b[g() % (len - 7)], &v, 8);
                }
                break;
            case 3:  // a 32-bit field (type tags, n_dims, value types)
                if (len >= 4) {
                    static const uint32_t vals[] = {0, 1, 3, 4, 5, 8, 9, 12, 13, 16, 42, 99, UINT32_MAX};
                    const uint32_t v = vals[g() % (sizeof(vals) / sizeof(vals[0]))];
                    memcpy(&b[g() % (len - 3)], &v, 4);
                }
                break;
            case 4:  // cut short
                if (len) b.resize(g() % len);
                break;
            case 5:  // extend with random bytes
                for (int i = 0, k = 1 + (int)(g() % 64); i < k; ++i) b.push_back((uint8_t)g());
                break;
            default:  // flip a bit in the header region
                if (len) b[g() % (len < 256 ? len : 256)] ^= (uint8_t)(1u << (g() % 8));
                break;
        }
    }
}

int main(int argc, char** argv) {
    if (argc < 4) {
        fprintf(stderr, "usage: %s <work-file> <iterations> <seed-file>...\n", argv[0]);
        return 2;
    }
    const char* work = argv[1];
    const long iters = atol(argv[2]);
    std::vector<std::vector<uint8_t>> seeds;
    for (int i = 3; i < argc; ++i) seeds.push_back(read_file(argv[i]));
    std::mt19937_64 g(0x9E3779B97F4A7C15ull);
    long opened = 0, refused = 0;
    char err[512];
    const char* keys[] = {"general.alignment", "general.architecture", "k", "a.list", ""};
    for (long it = 0; it < iters; ++it) {
        std::vector<uint8_t> b = seeds[it % seeds.size()];
        mutate(b, g);
        write_file(work, b);
        strata_gguf* m = nullptr;
        if (strata_cuda_gguf_open(work, &m, err, sizeof(err)) != STRATA_OK) {
            ++refused;
            if (m) return printf("open failed but returned a model\n"), 1;
            continue;
        }
        ++opened;
        strata_gguf_shard sh;
        for (int s = 0; s < strata_cuda_gguf_n_shards(m); ++s) strata_cuda_gguf_shard(m, s, &sh);
        const int64_t n = strata_cuda_gguf_tensor_count(m);
        for (int64_t i = 0; i < n; ++i) {
            strata_gguf_tensor t;
            if (strata_cuda_gguf_tensor(m, i, &t) != STRATA_OK) {
                strata_cuda_gguf_close(m);
                return printf("tensor %lld refused\n", (long long)i), 1;
            }
            int64_t found = -1;
            if (strlen(t.name) != t.name_len) {
                // a name holding a NUL byte: found (if at all) under its C-string prefix only
            } else if (strata_cuda_gguf_find(m, t.name, &found) != STRATA_OK || found != i) {
                strata_cuda_gguf_close(m);
                return printf("find(%s) = %lld, want %lld\n", t.name, (long long)found, (long long)i), 1;
            }
            const uint8_t* data = nullptr;
            uint64_t nbytes = 0;
            if (strata_cuda_gguf_tensor_data(m, i, &data, &nbytes, err, sizeof(err)) == STRATA_OK) {
                volatile uint8_t sink = 0;
                if (nbytes) sink ^= data[0] ^ data[nbytes - 1];  // the payload lies inside the mapping
                (void)sink;
            }
            strata_upload u;
            for (int64_t first : {(int64_t)0, (int64_t)1, (int64_t)-1})
                for (int64_t count : {(int64_t)-1, (int64_t)0, (int64_t)1, INT64_MAX})
                    if (strata_cuda_gguf_view(m, i, first, count, &u, err, sizeof(err)) == STRATA_OK && u.len) {
                        volatile uint8_t sink = u.bytes[0] ^ u.bytes[u.len - 1];
                        (void)sink;
                    }
        }
        strata_gguf_value v;
        for (const char* k : keys)
            if (strata_cuda_gguf_meta(m, k, &v) == STRATA_OK && v.type == STRATA_GGUF_STRING && v.str_len) {
                volatile char sink = v.str[0] ^ v.str[v.str_len - 1];
                (void)sink;
            }
        strata_cuda_gguf_close(m);
    }
    printf("ok %ld %ld\n", opened, refused);
    return 0;
}
