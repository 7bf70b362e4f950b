/* gen_expf_fix.c — build step: the table that makes the device's f32 exp equal
 * to the host C library's expf, bit for bit, on the max-shifted softmax domain
 * x in [-104, 0] (below -104 both are 0).
 *
 * strata-core's softmax and router (crates/strata-core/src/ops.rs:105-116,
 * crates/strata-core/src/moe.rs:57-68) call Rust's f32::exp, which is the
 * platform's expf. That function is not correctly rounded: measured on every
 * float of the domain, glibc's expf differs from the correctly rounded value
 * on 97,052 inputs, each within 1/256 ulp of a rounding midpoint (its error is
 * below 0.502 ulp). The device computes y = exp((double)x) and rounds it to
 * f32, which is correctly rounded unless y lies within a few double ulps of a
 * midpoint. So the device rule (expf_libm.cuh) is: if y is at least 2^-9 ulp
 * from the midpoint on its side, return the rounded y (there the C library
 * rounds correctly too: its misrounded inputs all lie within 2^-9.25 ulp of
 * one); otherwise look x up here and return the entry when there is one. The table holds every input of the domain where expf differs
 * from the correctly rounded value (found with the x87 long double expl), and
 * every input whose exact value lies within 16 double ulps of a midpoint
 * (where the device's own double exp may round either way), each with expf's
 * result.
 *
 * The entries are kept in an open-addressing hash table of 2^18 (key, value)
 * slots (key = |x|'s bits, value = expf's bits; Fibonacci hashing, linear
 * probing), so a lookup reads about one cache line; the longest probe any key
 * can take is recorded with it.
 *
 * The program then replays the device rule on every input of the domain, with
 * this host's double exp standing in for the device's, and fails unless all
 * 1,120,927,745 results equal expf's.
 *
 * usage: gen_expf_fix OUT.inc    (writes the C arrays the device code includes)
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define LO 0x80000000u /* -0.0 */
#define HI 0xC2D00000u /* -104.0 */
#define NTHREAD 8
#define SLOT_BITS 18
#define NSLOT (1u << SLOT_BITS)
#define EMPTY 0xFFFFFFFFu /* no key: |x| <= 0x42D00000 */

static float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* distance of y from the rounding midpoint on its side of r = round(y), in
 * ulps of r's neighbourhood (0 = on the midpoint, 0.5 = on r) */
static long double mid_dist(long double y, float r) {
    const uint32_t ur = u_of(r);
    const long double e = y - (long double)r;
    const float nb = f_of(e >= 0 ? ur + 1u : ur - 1u);
    const long double half = fabsl((long double)nb - (long double)r) / 2;
    return fabsl(fabsl(e) - half) / (2 * half);
}

typedef struct { uint32_t* in; uint32_t* out; size_t n, cap; uint32_t lo, hi; } part;

static void push(part* p, uint32_t in, uint32_t out) {
    if (p->n == p->cap) {
        p->cap = p->cap ? 2 * p->cap : 4096;
        p->in = realloc(p->in, p->cap * 4);
        p->out = realloc(p->out, p->cap * 4);
        if (!p->in || !p->out) { fprintf(stderr, "gen_expf_fix: out of memory\n"); exit(1); }
    }
    p->in[p->n] = in;
    p->out[p->n] = out;
    p->n++;
}

static void* collect(void* arg) {
    part* p = arg;
    for (uint32_t u = p->lo; u < p->hi; ++u) {
        const float x = f_of(u);
        const long double y = expl((long double)x);
        const float cr = (float)y;
        const uint32_t g = u_of(expf(x));
        const int hard = mid_dist(y, cr) < 16.0L / 536870912.0L; /* 16 double ulps, in f32 ulps */
        if (g != u_of(cr) || hard) push(p, u & 0x7FFFFFFFu, g);
    }
    return NULL;
}

/* the table, merged, and its hash slots */
static uint32_t* T_in;
static uint32_t* T_out;
static size_t T_n;
static uint32_t slot_key[NSLOT], slot_val[NSLOT];
static uint32_t max_probe; /* longest probe sequence of any key, hit or miss */

static uint32_t hash_of(uint32_t v) { return (v * 0x9E3779B1u) >> (32 - SLOT_BITS); }

/* the device rule of expf_libm.cuh, with the host's double exp */
static uint32_t device_rule(float x) {
    const double y = exp((double)x);
    const float r = (float)y;
    if (!(x <= 0.0f && x >= -104.0f)) return u_of(r);
    const uint32_t ur = u_of(r);
    const double e = y - (double)r;
    const float nb = f_of(e >= 0.0 ? ur + 1u : ur - 1u);
    const double half = 0.5 * fabs((double)nb - (double)r);
    if (fabs(fabs(e) - half) >= half * (1.0 / 256.0)) return ur;
    const uint32_t v = u_of(x) & 0x7FFFFFFFu;
    uint32_t h = hash_of(v);
    for (uint32_t p = 0; p < max_probe; ++p) {
        if (slot_key[h] == v) return slot_val[h];
        if (slot_key[h] == EMPTY) return ur;
        h = (h + 1) & (NSLOT - 1);
    }
    return ur;
}

typedef struct { uint32_t lo, hi; long long bad; uint32_t first; } check;

static void* verify(void* arg) {
    check* c = arg;
    for (uint32_t u = c->lo; u < c->hi; ++u) {
        const float x = f_of(u);
        if (device_rule(x) != u_of(expf(x))) {
            if (!c->bad) c->first = u;
            c->bad++;
        }
    }
    return NULL;
}

int main(int argc, char** argv) {
    if (argc != 2) { fprintf(stderr, "usage: gen_expf_fix OUT.inc\n"); return 2; }
    pthread_t th[NTHREAD];
    part parts[NTHREAD];
    memset(parts, 0, sizeof(parts));
    const uint32_t span = (HI + 1u - LO + NTHREAD - 1) / NTHREAD;
    for (int t = 0; t < NTHREAD; ++t) {
        parts[t].lo = LO + (uint32_t)t * span;
        parts[t].hi = t == NTHREAD - 1 ? HI + 1u : LO + (uint32_t)(t + 1) * span;
        pthread_create(&th[t], NULL, collect, &parts[t]);
    }
    for (int t = 0; t < NTHREAD; ++t) { pthread_join(th[t], NULL); T_n += parts[t].n; }
    T_in = malloc(T_n * 4);
    T_out = malloc(T_n * 4);
    size_t k = 0;
    for (int t = 0; t < NTHREAD; ++t) {  /* parts are in ascending input order */
        memcpy(T_in + k, parts[t].in, parts[t].n * 4);
        memcpy(T_out + k, parts[t].out, parts[t].n * 4);
        k += parts[t].n;
    }
    for (uint32_t h = 0; h < NSLOT; ++h) slot_key[h] = EMPTY;
    for (size_t i = 0; i < T_n; ++i) {
        uint32_t h = hash_of(T_in[i]);
        while (slot_key[h] != EMPTY) h = (h + 1) & (NSLOT - 1);
        slot_key[h] = T_in[i];
        slot_val[h] = T_out[i];
    }
    /* a probe from any slot ends at the first empty one: the longest run of
     * occupied slots (cyclically) plus that empty slot */
    for (uint32_t h = 0, run = 0, seen = 0; seen < 2 * NSLOT; ++seen, h = (h + 1) & (NSLOT - 1)) {
        run = slot_key[h] == EMPTY ? 0 : run + 1;
        if (run + 1 > max_probe) max_probe = run + 1;
    }

    check cs[NTHREAD];
    for (int t = 0; t < NTHREAD; ++t) {
        cs[t].lo = parts[t].lo; cs[t].hi = parts[t].hi; cs[t].bad = 0; cs[t].first = 0;
        pthread_create(&th[t], NULL, verify, &cs[t]);
    }
    long long bad = 0;
    for (int t = 0; t < NTHREAD; ++t) {
        pthread_join(th[t], NULL);
        if (cs[t].bad && !bad) fprintf(stderr, "gen_expf_fix: device rule differs from expf at 0x%08x\n", cs[t].first);
        bad += cs[t].bad;
    }
    if (bad) { fprintf(stderr, "gen_expf_fix: %lld inputs differ; no table written\n", bad); return 1; }

    FILE* f = fopen(argv[1], "w");
    if (!f) { perror(argv[1]); return 1; }
    fprintf(f, "// generated by gen_expf_fix.c from this host's expf: %zu entries, checked on every\n"
               "// float in [-104, 0] (the device rule with the host double exp equals expf on all).\n", T_n);
    fprintf(f, "#define STRATA_EXPF_FIX_ENTRIES %zu\n", T_n);
    fprintf(f, "constexpr int kExpfFixBits = %d;\nconstexpr uint32_t kExpfFixMaxProbe = %u;\n", SLOT_BITS, max_probe);
    fprintf(f, "static __device__ const uint2 kExpfFix[%u] = {", NSLOT);
    for (uint32_t h = 0; h < NSLOT; ++h)
        fprintf(f, "%s{0x%08xu,0x%08xu},", h % 6 ? "" : "\n", slot_key[h], slot_val[h]);
    fprintf(f, "\n};\n");
    if (fclose(f)) { perror(argv[1]); return 1; }
    printf("gen_expf_fix: %zu entries in %u slots (longest probe %u), all %u inputs match expf\n", T_n, NSLOT,
           max_probe, HI + 1u - LO);
    return 0;
}
