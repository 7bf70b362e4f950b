// Host check of strata_cuda_gguf_moe_layer (strata-rs_b200/csrc/gguf.cpp):
// the upload and layer-creation calls it makes are replaced by stand-ins
// that print what they were given, so the tensor lookup, the expert-range
// views and the layer description can be checked without a GPU.
//
// Usage: gguf_layer_check <model.gguf> <layer> <top_k> <expert_begin> <expert_end> <with_shared>
// Prints one "upload ..." line per tensor, one "desc ..." line, then "rc <status> <message>".
#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "../include/strata_gguf.h"

static std::string g_msg;
static int g_freed = 0;

extern "C" int strata_cuda_upload_many(strata_ctx*, const strata_upload* items, int64_t n, strata_weight** out) {
    for (int64_t i = 0; i < n; ++i) {
        const strata_upload& u = items[i];
        printf("upload %lld quant=%u n_expert=%lld rows=%lld cols=%lld len=%zu first=%u last=%u\n", (long long)i,
               u.quant, (long long)u.n_expert, (long long)u.rows, (long long)u.cols, u.len,
               u.len ? (unsigned)u.bytes[0] : 0u, u.len ? (unsigned)u.bytes[u.len - 1] : 0u);
        out[i] = reinterpret_cast<strata_weight*>((intptr_t)(i + 1));
    }
    return STRATA_OK;
}

static long long handle(const strata_weight* w) { return (long long)reinterpret_cast<intptr_t>(w); }

extern "C" int strata_cuda_moe_create(strata_ctx*, const strata_moe_desc* d, strata_moe** out) {
    printf("desc handles=%lld,%lld,%lld,%lld,%lld,%lld,%lld,%lld n_embd=%lld n_expert=%lld top_k=%lld n_ff=%lld "
           "n_ff_shexp=%lld begin=%lld end=%lld shared=%d\n",
           handle(d->router), handle(d->gate_exps), handle(d->up_exps), handle(d->down_exps), handle(d->gate_shexp),
           handle(d->up_shexp), handle(d->down_shexp), handle(d->gate_inp_shexp), (long long)d->n_embd,
           (long long)d->n_expert, (long long)d->top_k, (long long)d->n_ff, (long long)d->n_ff_shexp,
           (long long)d->expert_begin, (long long)d->expert_end, d->with_shared);
    *out = reinterpret_cast<strata_moe*>((intptr_t)99);
    return STRATA_OK;
}

extern "C" int strata_cuda_free_weight(strata_weight*) { return ++g_freed, STRATA_OK; }

namespace strata {
int report(strata_ctx*, int code, const char* msg) { return g_msg = msg, code; }
bool quant_on_device(uint32_t) { return true; }
}  // namespace strata

int main(int argc, char** argv) {
    if (argc != 7) return fprintf(stderr, "usage: %s model layer top_k begin end shared\n", argv[0]), 2;
    char err[512];
    strata_gguf* g = nullptr;
    int rc = strata_cuda_gguf_open(argv[1], &g, err, sizeof(err));
    if (rc) return printf("open %d %s\n", rc, err), 1;
    strata_moe* layer = nullptr;
    strata_weight* ws[8];
    strata_ctx* fake_ctx = reinterpret_cast<strata_ctx*>((intptr_t)7);  // never dereferenced by the stand-ins
    rc = strata_cuda_gguf_moe_layer(fake_ctx, g, atoll(argv[2]), atoll(argv[3]), atoll(argv[4]), atoll(argv[5]),
                                    atoi(argv[6]), &layer, ws);
    printf("rc %d %s\n", rc, g_msg.c_str());
    strata_cuda_gguf_close(g);
    return 0;
}
