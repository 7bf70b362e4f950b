// Host check of the upload staging plan (strata-rs_b200/csrc/staging.h):
// random lists of byte ranges (empty ones, ranges smaller and larger than a
// chunk, ranges that end exactly on a chunk boundary) are pushed through
// stage_plan / stage_fill with a small chunk and split among 8 "threads" the
// way the upload splits a chunk; every destination must come out equal to its
// source, every piece must stay inside its segment and its chunk, and the
// chunks must be full except the last. copy_host (the threaded host copy of
// large results) is checked on sizes around its thresholds with unaligned
// ends. Prints "ok" and exits 0, or names the first failure and exits 1.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "staging.h"

using namespace strata;

static int check(std::mt19937_64& g, size_t cap, int nseg_max) {
    std::uniform_int_distribution<int> nseg_d(0, nseg_max);
    const int nseg = nseg_d(g);
    std::vector<std::vector<uint8_t>> src(nseg), dst(nseg);
    std::vector<StageSeg> segs(nseg);
    size_t total = 0;
    for (int i = 0; i < nseg; ++i) {
        size_t n;
        switch (g() % 5) {
            case 0: n = 0; break;
            case 1: n = cap; break;
            case 2: n = 1 + g() % (cap / 3 + 1); break;
            case 3: n = cap * (1 + g() % 3) - g() % 2; break;
            default: n = 1 + g() % (4 * cap); break;
        }
        src[i].resize(n);
        for (auto& b : src[i]) b = (uint8_t)g();
        dst[i].assign(n, 0xEE);
        segs[i] = {dst[i].data(), src[i].data(), n};
        total += n;
    }
    std::vector<uint8_t> stage(cap);
    std::vector<StagePiece> pieces;
    StageCursor cur;
    size_t streamed = 0;
    for (int chunk = 0;; ++chunk) {
        const size_t len = stage_plan(segs.data(), nseg, cur, cap, pieces);
        if (!len) break;
        if (len > cap) return printf("chunk %d holds %zu > %zu bytes\n", chunk, len, cap), 1;
        if (len < cap && streamed + len != total) return printf("short chunk %d before the end\n", chunk), 1;
        size_t covered = 0;
        for (const StagePiece& p : pieces) {
            if (p.n == 0 || p.off != covered || p.off + p.n > len || p.seg_off + p.n > segs[p.seg].n)
                return printf("bad piece in chunk %d\n", chunk), 1;
            covered += p.n;
        }
        if (covered != len) return printf("chunk %d pieces cover %zu of %zu\n", chunk, covered, len), 1;
        std::fill(stage.begin(), stage.end(), 0xCD);
        const int T = 8;
        const size_t part = (len + T - 1) / T;
        for (int t = 0; t < T; ++t) {
            const size_t a = t * part, b = a + part < len ? a + part : len;
            if (a < b) stage_fill(pieces, segs.data(), stage.data(), a, b);
        }
        for (const StagePiece& p : pieces) memcpy(segs[p.seg].dst + p.seg_off, stage.data() + p.off, p.n);
        streamed += len;
    }
    if (streamed != total) return printf("streamed %zu of %zu bytes\n", streamed, total), 1;
    for (int i = 0; i < nseg; ++i)
        if (src[i] != dst[i]) return printf("segment %d differs\n", i), 1;
    return 0;
}

// copy_host over sizes on both sides of its thresholds and unaligned ends.
static int check_copy(std::mt19937_64& g) {
    const size_t sizes[] = {0, 1, 63, 4096, (size_t(2) << 20) - 1, size_t(2) << 20, (size_t(2) << 20) + 1,
                            (size_t(3) << 20) + 77, (size_t(9) << 20) + 5, (size_t(17) << 20) - 3};
    std::vector<size_t> all(sizes, sizes + sizeof(sizes) / sizeof(sizes[0]));
    for (int i = 0; i < 24; ++i) all.push_back((size_t(2) << 20) + g() % (size_t(15) << 20));
    for (size_t n : all) {
        const size_t so = g() % 64, dof = g() % 64;
        std::vector<uint8_t> src(n + so), dst(n + dof + 64, 0xAB);
        for (auto& b : src) b = (uint8_t)g();
        copy_host(dst.data() + dof, src.data() + so, n);
        if (n && memcmp(dst.data() + dof, src.data() + so, n) != 0) return printf("copy_host(%zu) differs\n", n), 1;
        for (size_t i = 0; i < dof; ++i)
            if (dst[i] != 0xAB) return printf("copy_host(%zu) wrote before dst\n", n), 1;
        for (size_t i = dof + n; i < dst.size(); ++i)
            if (dst[i] != 0xAB) return printf("copy_host(%zu) wrote past dst\n", n), 1;
    }
    return 0;
}

// CopyPool: the same property over consecutive copies through one pool (the
// workers persist between calls), including sizes under its threshold.
static int check_pool(std::mt19937_64& g) {
    CopyPool pool;
    for (int i = 0; i < 40; ++i) {
        const size_t n = i % 4 == 0 ? g() % (CopyPool::kMin + 1) : CopyPool::kMin + g() % (size_t(12) << 20);
        const size_t so = g() % 64, dof = g() % 64;
        std::vector<uint8_t> src(n + so), dst(n + dof + 64, 0xAB);
        for (auto& b : src) b = (uint8_t)g();
        if (i % 3 == 0) pool.prime();
        pool.copy(dst.data() + dof, src.data() + so, n);
        if (n && memcmp(dst.data() + dof, src.data() + so, n) != 0) return printf("pool.copy(%zu) differs\n", n), 1;
        for (size_t k = 0; k < dof; ++k)
            if (dst[k] != 0xAB) return printf("pool.copy(%zu) wrote before dst\n", n), 1;
        for (size_t k = dof + n; k < dst.size(); ++k)
            if (dst[k] != 0xAB) return printf("pool.copy(%zu) wrote past dst\n", n), 1;
    }
    return 0;
}

// CopyPool::copy2d: `height` rows of `width` bytes between pitched buffers
// land exactly, and nothing between or past the rows is written (row
// lengths over and under the threshold, one row to a few, parts that start
// and end inside rows).
static int check_pool_2d(std::mt19937_64& g) {
    CopyPool pool;
    for (int i = 0; i < 40; ++i) {
        const size_t h = 1 + g() % 9;
        const size_t w = i % 4 == 0 ? g() % 4096 : (CopyPool::kMin / h) + g() % (size_t(2) << 20);
        const size_t sp = w + g() % 200, dp = w + g() % 200;
        std::vector<uint8_t> src(sp * h + 64), dst(dp * h + 64, 0xAB);
        for (auto& b : src) b = (uint8_t)g();
        const size_t so = g() % 64;
        if (i % 3 == 0) pool.prime();
        pool.copy2d(dst.data(), dp, src.data() + so, sp, w, h);
        for (size_t r = 0; r < h; ++r) {
            if (w && memcmp(dst.data() + r * dp, src.data() + so + r * sp, w) != 0)
                return printf("pool.copy2d(%zu x %zu) row %zu differs\n", h, w, r), 1;
            const size_t end = r + 1 < h ? (r + 1) * dp : dst.size();
            for (size_t k = r * dp + w; k < end; ++k)
                if (dst[k] != 0xAB) return printf("pool.copy2d(%zu x %zu) wrote past row %zu\n", h, w, r), 1;
        }
    }
    return 0;
}

int main() {
    std::mt19937_64 g(20261202);
    if (check_copy(g)) return 1;
    if (check_pool(g)) return 1;
    if (check_pool_2d(g)) return 1;
    for (size_t cap : {size_t(1), size_t(7), size_t(64), size_t(1000), size_t(4096)})
        for (int it = 0; it < 300; ++it)
            if (check(g, cap, it % 3 == 0 ? 3 : 40)) return printf("cap %zu case %d\n", cap, it), 1;
    printf("ok\n");
    return 0;
}
