// Quantised GEMV on the sm_100a tensor cores: out[t][r] = sum_k W[r][k] * x[t][k]
// for up to 8 input vectors, weights streamed once from HBM.
//
// Reference: dot_*_b / gemv_rows_batch / gemv_multi_batch, src/kernels.c:323-736
// (one weight sweep serves all n <= GEMV_MAX_B vectors).  The block formats
// and their dequantisation are those of include/quant.h:14-62 and
// src/quant.c:86-182.
//
// Data path.  Weights are repacked once at load time from GGUF super-blocks
// into 16-row tiles whose bytes land directly in mma.sync A-fragment order
// (the byte count of every format is unchanged, except 2 B more per IQ4_XS
// row and super-block for its expanded sub-block scales).  Two tensor-core paths:
//  * IQ4_XS (93 % of the model's bytes): int8 mma m16n8k32.  Each code is
//    looked up as its int8 table value by byte permutes; the activations are
//    three balanced int8 digits per element after a power-of-two scale per
//    256-column block (~23 significant bits), so every sub-block dot product
//    is an exact int32, and the 6-bit sub-block scales are applied in int32 by
//    summation by parts along the mma accumulator chain.
//  * Q4_K / Q5_K / Q6_K / Q8_0: fp16 mma m16n8k16.  Each code becomes an
//    *exact* fp16 integer (the 1024+q exponent trick); the activations are
//    split into fp16 hi + lo halves after a power-of-two scale per block (~22
//    significant bits), the products are exact in the fp32 accumulator, and
//    per-32 / per-16 block scales are applied to each sub-block's fp32 sums.
// Either way results carry fp32-level error.
//
// Pipeline.  Two persistent CTAs of 8 warps per SM.  Every warp streams its
// own (pair of tiles x 256 columns) stages of contiguous repacked bytes into
// a private shared-memory ring with cp.async.bulk and mbarrier completion,
// refilling a slot as soon as it has decoded it (~140 KB in flight per SM),
// and decodes / runs the MMAs from shared memory.  The flattened (tile pair, block) stage
// space of all fused matrices is split evenly over every consumer warp of
// the grid (stream-K); a tile pair split across warps is finished by the last
// contributing warp, which sums the partials in warp order (deterministic).
// Programmatic dependent launch lets the producer prefetch weights while the
// previous kernel on the stream finishes.
//
// mma k-index <-> element mapping, shared by every format and by the
// activation fragments: within the 16-element step s of a 32-element
// sub-block, thread c of a quad holds elements 16s+4c .. 16s+4c+3;
// (4c, 4c+1) form register 0/1 (k = 2c, 2c+1) and (4c+2, 4c+3) register 2/3
// (k = 2c+8, 2c+9).
#include "qb_common.cuh"
#include "qb_kernels.h"
#include "qb_xprep.cuh"
#include "qb_iq4.cuh"
#include "qb_refmath.cuh"

namespace {

constexpr uint32_t H1152x2 = 0x64806480u;   // half2(1152, 1152) = 1024 + 128
constexpr uint32_t H1024x2 = 0x64006400u;   // half2(1024, 1024)
constexpr uint32_t H1056x2 = 0x64206420u;   // half2(1056, 1056) = 1024 + 32
constexpr uint32_t C64 = 0x64646464u;
constexpr int kConsumers = 8;                // warps per CTA (each streams its own weights)
constexpr int kThreads = kConsumers * 32;
#ifndef QB_QMV_CTAS
#define QB_QMV_CTAS 2
#endif
constexpr int kCtasPerSm = QB_QMV_CTAS;
// ring budget per CTA: 80 KB gives IQ4_XS a 2-stage ring per warp (141 KB in
// flight per SM, well above what HBM latency needs) and leaves the rest of the
// SM's shared memory to L1
#ifndef QB_QMV_SMEM_KB
#define QB_QMV_SMEM_KB 80
#endif
constexpr int kSmemBudget = QB_QMV_SMEM_KB * 1024;   // per CTA
#ifndef QB_QMV_MIN_STAGES
#define QB_QMV_MIN_STAGES 4
#endif
constexpr int kMinStagesPerWarp = QB_QMV_MIN_STAGES;
constexpr int kLocalPairs = 64;             // pairs one CTA's stage range may touch (else no level 1)
constexpr int kRingOff = 512;                // full barriers (8 warps x 8 slots x 8 B), then the rings
constexpr int kSsMax = 160;                  // deferred-norm sums prefetched per warp (N * K / 256)

// 4 unsigned bytes -> two half2 (1024 + b0, 1024 + b1), (1024 + b2, 1024 + b3)
__device__ __forceinline__ void bytes_to_h2(uint32_t u, uint32_t& h01, uint32_t& h23) {
    h01 = prmt(u, C64, 0x5140u);
    h23 = prmt(u, C64, 0x7362u);
}

template <int NT>
__device__ __forceinline__ void zero(float (&a)[NT][4]) {
#pragma unroll
    for (int c = 0; c < NT; ++c) a[c][0] = a[c][1] = a[c][2] = a[c][3] = 0.f;
}

template <int NT>
__device__ __forceinline__ void load_b(uint2 (&b)[NT], const uint2* __restrict__ xf, int lane) {
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) b[ct] = __ldg(xf + ct * 32 + lane);
}

template <int NT>
__device__ __forceinline__ void mma_nt(float (&cs)[NT][4], const uint32_t (&a)[4], const uint2 (&b)[NT]) {
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) mma_16816(cs[ct], a, b[ct].x, b[ct].y);
}

// the same with a zero accumulator input
template <int NT>
__device__ __forceinline__ void mma_nt_z(float (&cs)[NT][4], const uint32_t (&a)[4], const uint2 (&b)[NT]) {
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) mma_16816_z(cs[ct], a, b[ct].x, b[ct].y);
}

template <int NT>
__device__ __forceinline__ void scale_acc(float (&ab)[NT][4], const float (&cs)[NT][4], float dg, float dg8) {
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) {
        ab[ct][0] = fmaf(dg, cs[ct][0], ab[ct][0]);
        ab[ct][1] = fmaf(dg, cs[ct][1], ab[ct][1]);
        ab[ct][2] = fmaf(dg8, cs[ct][2], ab[ct][2]);
        ab[ct][3] = fmaf(dg8, cs[ct][3], ab[ct][3]);
    }
}

template <int NT>
__device__ __forceinline__ int col_token(int ct, int col) {
    return NT == 1 ? (col & 3) : col;
}

// ------------------------- per-format stage processors ------------------------
// A stage is (tile pair, one 256-column block); u points at the pair's bytes in
// shared memory (tile 2p, then tile 2p+1).  ab[t] accumulates, for tile t,
// sum over sub-blocks of (block scale * tensor-core partial); mt[t] collects
// terms that are not scaled by the activation scale (Q4_K / Q5_K mins).

// IQ4_XS tile-block: qs 2048 B (4 chunks x 32 lanes x 16 B), then 16 rows x 8
// int8 sub-block scale differences (ls_j - ls_{j+1} for j < 7, ls_7 - 32: the
// factors of the summation by parts below), then 16 rows x the fp16 d.
constexpr int kIq4Dl = 2048;
constexpr int kIq4D = 2048 + 16 * 8;
constexpr int kIq4Tile = kIq4D + 16 * 2;
static_assert(kIq4Tile == qb_unit_bytes(QB_IQ4_XS) && kIq4Tile % 16 == 0, "IQ4_XS tile-block layout");

// ---- IQ4_XS on the int8 tensor-core path (mma m16n8k32 s8 -> s32) ----
// Codes become the int8 values of kvalues_iq4nl (src/quant.c:30-32) as the
// sum of two byte-permute lookups (iq4_pq), each fed to its own mma; the activations arrive as three
// balanced int8 digits per token (X = 65536 d0 + 256 d1 + d2, xprep), so
// every sub-block dot product is exact in int32.  The same repacked tile
// layout as above serves both paths: the word of (row, sub-block) holds qs
// bytes 4c..4c+3, i.e. elements 4c..4c+3 (low nibbles) and 16+4c..16+4c+3
// (high nibbles), which is exactly the k-range of mma registers a0/a2 of
// thread c; the k order inside a register is (4c, 4c+16, 4c+1, 4c+17) and
// (4c+2, 4c+18, 4c+3, 4c+19), matched by the digit fragments.
//
// Columns of the n8 tiles: tile 0 = (token c: d0, d1), tile 1 = (token c: d2,
// token c+4: d2), tile 2 = (token c+4: d0, d1); NTI = 2 serves N <= 4.
//
// Sub-block scales by summation by parts: the mma chains its accumulator, so
// after sub-block j it holds R_j = sum_{i<=j} C_i, and
// sum_j s_j C_j = sum_{j<7} (s_j - s_{j+1}) R_j + s_7 R_7 with s_j = ls_j - 32.
// B fragments of sub-block sb of a block
template <int NTI>
__device__ __forceinline__ void load_bq(uint2 (&b)[NTI], const uint2* __restrict__ xq, int sb, int lane) {
#pragma unroll
    for (int nt = 0; nt < NTI; ++nt) b[nt] = __ldg(xq + (sb * NTI + nt) * 32 + lane);
}

// v[t][r][k]: d * (sum over the super-block) for tile t, row g + 8r, token c + 4k.
// bb holds the B fragments of sub-blocks 0 and 1 on entry; loads run two
// sub-blocks ahead, so on return bb holds sub-blocks 0 and 1 of xq_next.
template <int NTI>
__device__ __forceinline__ void stage_iq4_i8(const uint8_t* u, const uint2* __restrict__ xq,
                                             const uint2* __restrict__ xq_next, int lane, uint2 (&bb)[2][NTI],
                                             float (&v)[2][2][2]) {
    const int g = lane >> 2;
    float d[2][2];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 2; ++r) d[t][r] = h2f_bits(lds16(u + t * kIq4Tile + kIq4D + (g + 8 * r) * 2));
    int R[2][NTI][4], acc[2][NTI][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int nt = 0; nt < NTI; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) R[t][nt][i] = acc[t][nt][i] = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint4 q0 = lds128(u + p * 512 + lane * 16);
        const uint4 q1 = lds128(u + kIq4Tile + p * 512 + lane * 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int sb = 2 * p + h;
            uint2 bq[NTI];
#pragma unroll
            for (int nt = 0; nt < NTI; ++nt) bq[nt] = bb[h][nt];
            if (sb < 6) load_bq<NTI>(bb[h], xq, sb + 2, lane);
            else load_bq<NTI>(bb[h], xq_next, sb - 6, lane);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const uint4& q = t ? q1 : q0;
                uint32_t pa[4], qa[4];
                iq4_pq(h ? q.z : q.x, pa[0], pa[2], qa[0], qa[2]);   // row g
                iq4_pq(h ? q.w : q.y, pa[1], pa[3], qa[1], qa[3]);   // row g + 8
#pragma unroll
                for (int nt = 0; nt < NTI; ++nt) {
                    mma_16832_s8(R[t][nt], pa, bq[nt].x, bq[nt].y);
                    mma_16832_s8(R[t][nt], qa, bq[nt].x, bq[nt].y);
                }
                const uint8_t* dl = u + t * kIq4Tile + kIq4Dl + g * 8 + sb;
                const int s_g = lds_s8(dl), s_g8 = lds_s8(dl + 64);
#pragma unroll
                for (int nt = 0; nt < NTI; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (NTI == 2 && nt == 1 && (i & 1)) continue;   // unused column
                        acc[t][nt][i] += ((i & 2) ? s_g8 : s_g) * R[t][nt][i];
                    }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            v[t][r][0] = fmaf((float)acc[t][0][2 * r], 65536.f, fmaf((float)acc[t][0][2 * r + 1], 256.f,
                                                                     (float)acc[t][1][2 * r])) * d[t][r];
            v[t][r][1] = NTI == 3 ? fmaf((float)acc[t][NTI - 1][2 * r], 65536.f,
                                         fmaf((float)acc[t][NTI - 1][2 * r + 1], 256.f,
                                              (float)acc[t][1][2 * r + 1])) * d[t][r]
                                  : 0.f;
        }
}

// Q8_0: tile-block = 8 units of 544 B (32 columns: 16 rows x 32 qs in lane
// order [row g s0][row g8 s0][row g s1][row g8 s1], then 16 x fp16 d).
constexpr int kQ8Tile = 8 * 544;
template <int NT>
__device__ __forceinline__ void stage_q8_0(const uint8_t* u, const uint2* __restrict__ xf, int lane,
                                           float (&ab)[2][NT][4], float (&)[2][NT][4]) {
    const int g = lane >> 2;
#pragma unroll 2
    for (int sb = 0; sb < 8; ++sb) {
        float cs[2][NT][4];
        zero<NT>(cs[0]);
        zero<NT>(cs[1]);
        uint32_t a[2][2][4];
        float dd[2][2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const uint8_t* un = u + t * kQ8Tile + sb * 544;
            const uint4 q = lds128(un + lane * 16);
            const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                bytes_to_h2(w[2 * s], a[t][s][0], a[t][s][2]);
                bytes_to_h2(w[2 * s + 1], a[t][s][1], a[t][s][3]);
#pragma unroll
                for (int i = 0; i < 4; ++i) a[t][s][i] = hsub2_u32(a[t][s][i], H1152x2);
            }
            const uint32_t dw = lds32(un + 512 + (g & ~1) * 2);                   // rows g&~1, g|1
            const uint32_t dw8 = lds32(un + 512 + ((g + 8) & ~1) * 2);
            dd[t][0] = h2f_bits(g & 1 ? dw >> 16 : dw);
            dd[t][1] = h2f_bits(g & 1 ? dw8 >> 16 : dw8);
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            uint2 b[NT];
            load_b<NT>(b, xf + (sb * 2 + s) * NT * 32, lane);
#pragma unroll
            for (int t = 0; t < 2; ++t) mma_nt<NT>(cs[t], a[t][s], b);
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) scale_acc<NT>(ab[t], cs[t], dd[t][0], dd[t][1]);
    }
}

// Q4_K / Q5_K: w = d*sc*q - dmin*m -> d*sc*sum(q x) - dmin*m*sum(x)
// (src/kernels.c:414-510; get_scale_min_k4 include/quant.h:21-29).
// Tile-block: qs 2048 B (chunk j: [row g s0][row g s1][row g8 s0][row g8 s1]
// of bytes 32j + 16s + 4c..), [qh 512 B (Q5_K): [row g s0][row g s1][row g8 s0]
// [row g8 s1] of qh bytes 16s + 4c..], then 16 rows x [d dmin scales(12)].
__device__ __forceinline__ void k4_scale_min(const uint8_t* s12, int j, float& sc, float& m) {
    uint32_t d, mm;
    if (j < 4) {
        d = s12[j] & 63;
        mm = s12[j + 4] & 63;
    } else {
        d = (s12[j + 4] & 0xF) | ((s12[j - 4] >> 6) << 4);
        mm = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4);
    }
    sc = small_u2f(d);
    m = small_u2f(mm);
}

template <int NT, bool Q5>
__device__ __forceinline__ void stage_qk(const uint8_t* u, const uint2* __restrict__ xf, const float* __restrict__ xsum_blk,
                                         int xsum_stride, int lane, float (&ab)[2][NT][4], float (&mt)[2][NT][4]) {
    const int g = lane >> 2, c = lane & 3;
    constexpr int TB = Q5 ? 16 * 176 : 16 * 144;
    constexpr int SC = Q5 ? 2560 : 2048;
#pragma unroll 1
    for (int t = 0; t < 2; ++t) {
        const uint8_t* ut = u + t * TB;
        const uint4 hg = lds128(ut + SC + g * 16);
        const uint4 hg8 = lds128(ut + SC + (g + 8) * 16);
        const float dg = h2f_bits(hg.x), dmg = h2f_bits(hg.x >> 16);
        const float dg8 = h2f_bits(hg8.x), dmg8 = h2f_bits(hg8.x >> 16);
        uint8_t s12g[12], s12g8[12];
        {
            const uint32_t a[3] = {hg.y, hg.z, hg.w}, b[3] = {hg8.y, hg8.z, hg8.w};
#pragma unroll
            for (int i = 0; i < 12; ++i) {
                s12g[i] = (uint8_t)(a[i >> 2] >> (8 * (i & 3)));
                s12g8[i] = (uint8_t)(b[i >> 2] >> (8 * (i & 3)));
            }
        }
        uint4 qh = make_uint4(0, 0, 0, 0);
        if (Q5) qh = lds128(ut + 2048 + lane * 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 q = lds128(ut + j * 512 + lane * 16);
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
                const int sb = 2 * j + hi;
                float cs[NT][4];
                zero<NT>(cs);
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    uint32_t ug = ((s ? q.y : q.x) >> (4 * hi)) & 0x0F0F0F0Fu;
                    uint32_t ug8 = ((s ? q.w : q.z) >> (4 * hi)) & 0x0F0F0F0Fu;
                    if (Q5) {
                        ug |= (((s ? qh.y : qh.x) >> sb) & 0x01010101u) << 4;
                        ug8 |= (((s ? qh.w : qh.z) >> sb) & 0x01010101u) << 4;
                    }
                    uint32_t a[4];
                    bytes_to_h2(ug, a[0], a[2]);
                    bytes_to_h2(ug8, a[1], a[3]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[i] = hsub2_u32(a[i], H1024x2);
                    uint2 b[NT];
                    load_b<NT>(b, xf + (sb * 2 + s) * NT * 32, lane);
                    mma_nt<NT>(cs, a, b);
                }
                float scg, mg, scg8, mg8;
                k4_scale_min(s12g, sb, scg, mg);
                k4_scale_min(s12g8, sb, scg8, mg8);
                scale_acc<NT>(ab[t], cs, dg * scg, dg8 * scg8);
#pragma unroll
                for (int ct = 0; ct < NT; ++ct)
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int col = 2 * c + i;
                        const bool is_lo = NT == 1 ? (col >= 4) : (ct == 1);
                        if (!is_lo) {
                            const float xs = xsum_blk[col_token<NT>(ct, col) * xsum_stride + sb];
                            mt[t][ct][i] -= dmg * mg * xs;
                            mt[t][ct][2 + i] -= dmg8 * mg8 * xs;
                        }
                    }
            }
        }
    }
}

// Q6_K tile-block: lo plane 2048 B (chunk qc: word i = group 4qc+i, nibbles
// 0..3 = row g elements 4c..4c+3, 4..7 = row g8), hi plane 1024 B (word per
// group pair: byte j bits 4-5/6-7 = even/odd member of the first group, 0-1/
// 2-3 of the second), scales 16 rows x 16 bytes (int8 scale + 128), d 16 x fp16.
constexpr int kQ6Tile = 16 * 210;
template <int NT>
__device__ __forceinline__ void stage_q6k(const uint8_t* u, const uint2* __restrict__ xf, int lane,
                                          float (&ab)[2][NT][4], float (&)[2][NT][4]) {
    const int g = lane >> 2;
#pragma unroll 1
    for (int t = 0; t < 2; ++t) {
        const uint8_t* ut = u + t * kQ6Tile;
        const uint4 sc_g = lds128(ut + 3072 + g * 16);
        const uint4 sc_g8 = lds128(ut + 3072 + (g + 8) * 16);
        const uint32_t dw = lds32(ut + 3328 + (g & ~1) * 2);
        const uint32_t dw8 = lds32(ut + 3328 + ((g + 8) & ~1) * 2);
        const float dg = h2f_bits(g & 1 ? dw >> 16 : dw), dg8 = h2f_bits(g & 1 ? dw8 >> 16 : dw8);
        const uint32_t scw_g[4] = {sc_g.x, sc_g.y, sc_g.z, sc_g.w};
        const uint32_t scw_g8[4] = {sc_g8.x, sc_g8.y, sc_g8.z, sc_g8.w};
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            const uint4 hq = lds128(ut + 2048 + ch * 512 + lane * 16);
            const uint32_t hw[4] = {hq.x, hq.y, hq.z, hq.w};
#pragma unroll
            for (int qc = 0; qc < 2; ++qc) {
                const uint4 lq = lds128(ut + (ch * 2 + qc) * 512 + lane * 16);
                const uint32_t lw[4] = {lq.x, lq.y, lq.z, lq.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int G = (ch * 2 + qc) * 4 + i;
                    const uint32_t h = hw[(G >> 1) & 3];
                    const bool Bg = G & 1;
                    const uint32_t he = Bg ? ((h << 4) & 0x30303030u) : (h & 0x30303030u);
                    const uint32_t ho = Bg ? ((h << 2) & 0x30303030u) : ((h >> 2) & 0x30303030u);
                    const uint32_t ev = (lw[i] & 0x0F0F0F0Fu) | he;
                    const uint32_t od = ((lw[i] >> 4) & 0x0F0F0F0Fu) | ho;
                    const uint32_t p01 = prmt(ev, od, 0x5140u);
                    const uint32_t p23 = prmt(ev, od, 0x7362u);
                    uint32_t a[4];
                    a[0] = hsub2_u32(prmt(p01, C64, 0x5140u), H1056x2);
                    a[2] = hsub2_u32(prmt(p01, C64, 0x7362u), H1056x2);
                    a[1] = hsub2_u32(prmt(p23, C64, 0x5140u), H1056x2);
                    a[3] = hsub2_u32(prmt(p23, C64, 0x7362u), H1056x2);
                    float cs[NT][4];
                    uint2 b[NT];
                    load_b<NT>(b, xf + G * NT * 32, lane);
                    mma_nt_z<NT>(cs, a, b);
                    // the scale byte u = sc + 128 as the float 2^23 + u, minus 2^23 + 128: sc, exactly
                    const uint32_t sel = 0x7650u | (uint32_t)(G & 3);
                    const float scg = __uint_as_float(prmt(scw_g[G >> 2], 0x4B000000u, sel)) - 8388736.0f;
                    const float scg8 = __uint_as_float(prmt(scw_g8[G >> 2], 0x4B000000u, sel)) - 8388736.0f;
                    scale_acc<NT>(ab[t], cs, dg * scg, dg8 * scg8);
                }
            }
        }
    }
}

__host__ __device__ constexpr int tile_block_bytes(int type) {
    return type == QB_IQ4_XS ? kIq4Tile
         : type == QB_Q8_0   ? kQ8Tile
         : type == QB_Q6_K   ? kQ6Tile
         : type == QB_Q4_K   ? 16 * 144
         : type == QB_Q5_K   ? 16 * 176
         : 0;
}

// ------------------------------- the kernel ------------------------------------

struct TpK {
    int np, rank;                // peers, this rank
    int gather;                  // 1: rows to every peer + wait; 0: tagged partial sums into part
    uint2* part;                 // partial mode: 2 slots of [.][ldo] (value, tag), slot = sequence parity
    long long part_slot;         // words per slot
    long long delta[QB_TP_MAX - 1];   // byte offset from a local arena address to the same address of peer i
    unsigned* flags;             // [QB_TP_MAX] in the shared arena: the last sequence number seen from each rank
    unsigned* done;              // warps of the grid that finished (zero between launches)
    unsigned* seq;               // this rank's count of TP launches
    unsigned* err;
};

struct QmvK {
    QSeg seg[QB_MAX_SEG];
    int pair0[QB_MAX_SEG + 1];   // first tile pair of each segment; pair0[nseg] = total pairs
    int nseg;
    int K, nb, N;
    int S;                       // total stages = pairs * nb (fits 32 bits for every launch)
    int Wt;                      // consumer warps in the grid
    int stages_per_warp_ring;    // ring depth
    const uint2* xfrag;
    const float* xscale;
    const float* xsum;
    const uint2* xq;             // int8 digit fragments (IQ4_XS int8 path)
    const float* xqscale;
    int accumulate;
    int row_lo, row_hi;
    float* partial;              // [Wt][2][32][8] warp partials of split pairs
    float* gpartial;             // [Wt / group + 1][2][32][8] group partials
    unsigned* counters;          // [pairs]
    int group;                   // warps combined in shared memory before the device-wide combine
    unsigned* err;
    // tensor parallelism (QbTp): every stored output value also goes to the
    // same address of each peer's buffer (dst + tp_delta[i]), then the grid's
    // last warp exchanges a sequence number with the peers (cross-rank barrier)
    TpK tp;
    // deferred RMSNorm of the input (QbInNorm), in_ss == nullptr: none
    const float* in_ss;
    float in_eps;
    // fused preparation of the next input (QbEpi)
    int epi;                     // QB_EPI_*
    unsigned* bcnt;              // [output blocks] pair arrivals, zero between launches
    const float* epi_w;
    float* epi_ss;
    float* epi_h;
    long long epi_ldh;
    int epi_K;                   // columns of the next input (= this launch's output rows, or half of them)
    int epi_what;
    QbXBuf epi_xb;
};

// stage ranges: warp w owns [S*w/Wt, S*(w+1)/Wt); the grid guarantees Wt <= S,
// so every warp owns at least one stage.  S * Wt < 2^31 for every launch.
__device__ __forceinline__ int warp_s0(int S, int Wt, int w) { return (int)((unsigned)(S * w) / (unsigned)Wt); }
__device__ __forceinline__ int stage_owner(int S, int Wt, int s) {
    return (int)((unsigned)((s + 1) * Wt - 1) / (unsigned)S);
}

// Next-input preparation for the 256-row output block blk, by the warp that
// finished its last tile pair: per token, 8 values per lane (elements
// 4 lane .. 4 lane + 3 and 128 + 4 lane ..) of src (h, or the residual x
// times the norm weight w), then the fragments.  Four tokens at a time, so
// that their load / shuffle chains overlap (tokens N..3 of a group are
// computed too and land in the unused token columns; every buffer holds
// QB_MAX_TOK tokens).  Not inlined, and given plain values, so that the GEMV
// main loop keeps its registers.
__device__ __noinline__ void block_emit(const float* __restrict__ src, long long ld, const float* __restrict__ w,
                                        float* __restrict__ ss_out, int blk, int N, int K, QbXBuf xb, int what,
                                        int lane) {
    const int nbo = K >> 8;
    for (int t0 = 0; t0 < N; t0 += 4) {
        float v[4][8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float* x = src + (size_t)(t0 + k) * ld + (size_t)blk * 256;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(x + h * 128 + 4 * lane));
                v[k][4 * h + 0] = a.x; v[k][4 * h + 1] = a.y; v[k][4 * h + 2] = a.z; v[k][4 * h + 3] = a.w;
            }
        }
        if (w) {
            float wv[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(w + (size_t)blk * 256 + h * 128 + 4 * lane));
                wv[4 * h + 0] = a.x; wv[4 * h + 1] = a.y; wv[4 * h + 2] = a.z; wv[4 * h + 3] = a.w;
            }
            float ss[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                ss[k] = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) ss[k] = fmaf(v[k][i], v[k][i], ss[k]);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1)
#pragma unroll
                for (int k = 0; k < 4; ++k) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], o);
            if (lane == 0)
#pragma unroll
                for (int k = 0; k < 4; ++k) ss_out[(t0 + k) * nbo + blk] = ss[k];
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int i = 0; i < 8; ++i) v[k][i] = __fmul_rn(v[k][i], wv[i]);
        }
        xprep_emit_g<4>(v, t0, blk, N, nbo, K, xb, what, lane);
    }
}

// 1 / rms of tokens 2c and 2c + 1 (c = lane & 3) from the producer's per-block
// sums of squares, in a fixed order: ss[t * nb + b], prefetched into s_ss at
// kernel start when N * nb <= kSsMax.  Not inlined: it runs once per pair.
__device__ __noinline__ void deferred_inv(const float* s_ss, const float* __restrict__ ss, int N, int nb, int K,
                                          float eps, int lane, float& i0, float& i1) {
    const bool pre = N * nb <= kSsMax;
    if (pre) {
        cp_async_wait_all();
        __syncwarp();
    }
    float sum[QB_MAX_TOK];
#pragma unroll
    for (int t = 0; t < QB_MAX_TOK; ++t) {
        sum[t] = 0.f;
        if (t < N)
            for (int b = lane; b < nb; b += 32) sum[t] += pre ? s_ss[t * nb + b] : __ldg(ss + (size_t)t * nb + b);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int t = 0; t < QB_MAX_TOK; ++t) sum[t] += __shfl_xor_sync(0xffffffffu, sum[t], o);
    const int t0 = 2 * (lane & 3), t1 = t0 + 1;
    i0 = i1 = 1.f;
#pragma unroll
    for (int t = 0; t < QB_MAX_TOK; ++t) {
        const float iv = 1.0f / sqrtf(sum[t] / (float)K + eps);
        if (t == t0) i0 = iv;
        if (t == t1) i1 = iv;
    }
}

// The final values of a tile pair, held by one warp (lanes with active ==
// false hold nothing): the deferred input norm, the store (or SwiGLU of the
// gate / up tiles), then the block-completion epilogue.
template <bool EPI, bool TP>
__device__ __forceinline__ void pair_final(const QmvK& p, int pair, float (&v)[2][4], bool active, int lane,
                                           const float* s_ss) {
    int si = 0;
#pragma unroll
    for (int s = 1; s < QB_MAX_SEG; ++s)
        if (s < p.nseg && pair >= p.pair0[s]) si = s;
    const QSeg& S = p.seg[si];
    const int lp = pair - p.pair0[si];
    const int g = lane >> 2, c = lane & 3;
    const int t0 = 2 * c, t1 = 2 * c + 1;
    if (EPI && p.in_ss) {
        float i0, i1;
        deferred_inv(s_ss, p.in_ss, p.N, p.nb, p.K, p.in_eps, lane, i0, i1);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[t][i] *= (i & 1) ? i1 : i0;
    }
    if (EPI && p.epi == QB_EPI_SWIGLU) {
        if (active)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = lp * 16 + g + ((i & 2) ? 8 : 0);
                const int tok = (i & 1) ? t1 : t0;
                if (tok < p.N) p.epi_h[(size_t)tok * p.epi_ldh + j] = __fmul_rn(silu_ref(v[0][i]), v[1][i]);
            }
    } else if (active) {
        // residual launches: every old value is loaded before the first store, so the
        // eight loads overlap instead of each waiting behind the previous store (the
        // stores may alias them, so the compiler keeps the order it is given)
        float prev[2][4];
        if (p.accumulate && !(TP && !p.tp.gather)) {
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int rr = lp * 32 + t * 16 + g + ((i & 2) ? 8 : 0);
                    const int tok = (i & 1) ? t1 : t0;
                    prev[t][i] = (tok < p.N && rr < S.rows && rr >= p.row_lo && rr < p.row_hi)
                                     ? __ldcg(S.out + (size_t)tok * S.ldo + rr)
                                     : 0.f;
                }
        }
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int rr = lp * 32 + t * 16 + g + ((i & 2) ? 8 : 0);
                const int tok = (i & 1) ? t1 : t0;
                if (tok < p.N && rr < S.rows && rr >= p.row_lo && rr < p.row_hi) {
                    float* dst = S.out + (size_t)tok * S.ldo + rr;
                    if (TP && !p.tp.gather) {
                        // partial sum of this rank as one 8-byte (value, tag) store, tag = this launch's
                        // sequence number: a peer that sees the tag has the value (no fence, no flag)
                        const unsigned sq = *(volatile const unsigned*)p.tp.seq;
                        uint2* w = p.tp.part + (size_t)(sq & 1u) * p.tp.part_slot + (size_t)tok * S.ldo + rr;
                        *w = make_uint2(__float_as_uint(v[t][i]), sq + 1u);
                        continue;
                    }
                    const float y = p.accumulate ? prev[t][i] + v[t][i] : v[t][i];
                    *dst = y;
                    if (TP && p.tp.gather)
                        for (int q = 0; q < p.tp.np; ++q)
                            *reinterpret_cast<float*>(reinterpret_cast<char*>(dst) + p.tp.delta[q]) = y;
                }
            }
    }
    if (!EPI || p.epi == QB_EPI_NONE) return;
    // block of 256 output rows complete: 8 pairs (16 for SwiGLU, whose pairs yield 16 rows of h)
    const int ppb = p.epi == QB_EPI_SWIGLU ? 16 : 8;
    const int blk = lp / ppb;
    // the warp's stores, then one acquire-release arrival (cumulative over the warp's stores)
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(p.bcnt + blk, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if ((int)old != ppb - 1) return;
    if (lane == 0) p.bcnt[blk] = 0u;   // ready for the next launch
    __syncwarp();
    if (p.epi == QB_EPI_SWIGLU)
        block_emit(p.epi_h, p.epi_ldh, nullptr, nullptr, blk, p.N, p.epi_K, p.epi_xb, p.epi_what, lane);
    else
        block_emit(S.out, S.ldo, p.epi_w, p.epi_ss, blk, p.N, p.epi_K, p.epi_xb, p.epi_what, lane);
}

// o[t][i], i = (row g tok 2c, row g tok 2c+1, row g8 tok 2c, row g8 tok 2c+1) of
// tile t; lanes with active == false hold nothing to store.
template <bool EPI, bool TP>
__device__ __forceinline__ void finish_pair(const QmvK& p, int pair, int gw, int s0, int s1, const float (&o)[2][4],
                                            bool active, int lane, unsigned* lcnt, int grp_pair0, const float* s_ss) {
    const int g = lane >> 2, c = lane & 3;
    const int t0 = 2 * c, t1 = 2 * c + 1;
    const int P0 = pair * p.nb, P1 = P0 + p.nb;
    float v[2][4];
    if (s0 <= P0 && s1 >= P1) {
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[t][i] = o[t][i];
        pair_final<EPI, TP>(p, pair, v, active, lane, s_ss);
        return;
    }
    // Split pair.  A contributor's piece is 0 if it started inside the pair
    // (the pair is its first), 1 if it started before (the pair is its last).
    auto pidx = [&](int t, int i) { return (t * 16 + g + ((i & 2) ? 8 : 0)) * 8 + ((i & 1) ? t1 : t0); };
    auto piece_of = [&](int first_warp) { return warp_s0(p.S, p.Wt, first_warp) >= P0 ? 0 : 1; };
    const int G = p.group;   // warps combined through shared memory first (8 = a CTA, 1 = none)
    const int w_first = stage_owner(p.S, p.Wt, P0), w_last = stage_owner(p.S, p.Wt, P1 - 1);
    const int grp = gw / G;
    const int lw_first = max(w_first, grp * G), lw_last = min(w_last, grp * G + G - 1);
    if (lw_first == lw_last) {
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[t][i] = o[t][i];
    } else {
        // level 1: the group's warps, block-scope ordering, last arrival sums in warp order
        float* slot = p.partial + ((size_t)gw * 2 + piece_of(gw)) * 256;
        if (active)
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int i = 0; i < 4; ++i) slot[pidx(t, i)] = o[t][i];
        __threadfence_block();
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(lcnt + (pair - grp_pair0), 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if ((int)old != lw_last - lw_first) return;
        __threadfence_block();
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[t][i] = 0.f;
        for (int w = lw_first; w <= lw_last; ++w) {
            const volatile float* sl = p.partial + ((size_t)w * 2 + piece_of(w)) * 256;
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int i = 0; i < 4; ++i) v[t][i] += sl[pidx(t, i)];
        }
    }
    const int g_first = w_first / G, g_last = w_last / G;
    if (g_first == g_last) {
        pair_final<EPI, TP>(p, pair, v, active, lane, s_ss);
        return;
    }
    // level 2: the groups, device-scope ordering, last arrival sums in group order
    float* gslot = p.gpartial + ((size_t)grp * 2 + piece_of(grp * G)) * 256;
    if (active)
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) gslot[pidx(t, i)] = v[t][i];
    // the warp barrier orders every lane's stores before lane 0's release (cumulative), and
    // the last arrival's acquire before every lane's loads: no full fences on this path
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(p.counters + pair, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if ((int)old != g_last - g_first) return;
    float sum[2][4] = {};
    for (int gg = g_first; gg <= g_last; ++gg) {
        const volatile float* sl = p.gpartial + ((size_t)gg * 2 + piece_of(gg * G)) * 256;
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) sum[t][i] += sl[pidx(t, i)];
    }
    if (lane == 0) p.counters[pair] = 0u;   // ready for the next launch
    pair_final<EPI, TP>(p, pair, sum, active, lane, s_ss);
}

// fp16 path: combine the hi/lo columns of the mma accumulators
template <int NT>
__device__ __forceinline__ void pair_out_f16(const float (&acc)[2][NT][4], float (&o)[2][4], bool& active, int lane) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i)
            o[t][i] = NT == 1 ? acc[t][0][i] + __shfl_xor_sync(0xffffffffu, acc[t][0][i], 2)
                              : acc[t][0][i] + acc[t][NT - 1][i];
    active = NT == 1 ? ((lane & 3) < 2) : true;
}

// int8 path: lane (g, c) holds tok[t][r][k] = (tile t, row g + 8r, token c + 4k);
// regroup to tokens (2c, 2c+1) per lane
template <int NT>
__device__ __forceinline__ void pair_out_i8(const float (&tok)[2][2][2], float (&o)[2][4], bool& active, int lane) {
    const int c = lane & 3, base = lane & ~3;
    const int src0 = base + ((2 * c) & 3), src1 = base + ((2 * c + 1) & 3);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float a0 = __shfl_sync(0xffffffffu, tok[t][r][0], src0);
            const float a1 = __shfl_sync(0xffffffffu, tok[t][r][0], src1);
            if (NT == 1) {
                o[t][2 * r] = a0;
                o[t][2 * r + 1] = a1;
            } else {
                const float b0 = __shfl_sync(0xffffffffu, tok[t][r][1], src0);
                const float b1 = __shfl_sync(0xffffffffu, tok[t][r][1], src1);
                o[t][2 * r] = (c >> 1) ? b0 : a0;
                o[t][2 * r + 1] = (c >> 1) ? b1 : a1;
            }
        }
    active = NT == 1 ? (c < 2) : true;
}

// Tensor parallelism: a warp that is done (its stores, peer stores included) arrives
// on its CTA's shared counter (acquire-release, so the CTA's last warp has
// observed every store of the CTA); that warp makes them visible system-wide
// and arrives on the device counter; the grid's last CTA publishes the
// launch's sequence number into its slot of every peer's flag array and
// waits, bounded, until every peer has published the same number into this
// rank's array.  The launch therefore ends only when all ranks' outputs have
// landed here.  A warp that gave up a wait never arrives, so the peers time
// out and record the error too.
__device__ __noinline__ void tp_arrive(TpK t, uint32_t s_arrive, int lane) {
    __syncwarp();
    if (lane != 0) return;
    unsigned old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;" : "=r"(old) : "r"(s_arrive) : "memory");
    if (old != kConsumers - 1) return;
    if (t.gather) __threadfence_system();   // the CTA's stores, peer stores included
    old = atom_add_acq_rel_gpu(t.done, 1u);
    if (old != gridDim.x - 1) return;
    *t.done = 0u;   // ready for the next launch
    const unsigned seq = *t.seq + 1u;
    *t.seq = seq;
    if (!t.gather) return;   // tagged partial sums: the reduction checks the tags
    for (int q = 0; q < t.np; ++q) {
        unsigned* slot = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(t.flags + t.rank) + t.delta[q]);
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slot), "r"(seq) : "memory");
    }
    for (int q = 0; q < t.np; ++q) {
        const int peer = q < t.rank ? q : q + 1;
        const unsigned* f = t.flags + peer;
        const unsigned long long t0 = global_ns();
        for (uint32_t it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if ((int)(v - seq) >= 0) break;
            if (peer_wait_over(it, t0, t.err, 4u)) return;
            __nanosleep(64);
        }
    }
}

// EPI: the launch has a deferred input norm or a next-input epilogue (QbInNorm,
// QbEpi); launches without either run the variant that has neither.
// TP: tensor-parallel launch (peer stores and the cross-rank barrier, QbTp).
template <int FMT, int NT, bool I8, bool EPI, bool TP>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) qmv_kernel(QmvK p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = tile_block_bytes(FMT);
    constexpr uint32_t STAGE = 2 * TB;
    const int R = p.stages_per_warp_ring;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem) + warp * 8;
    uint8_t* ring = smem + kRingOff + (size_t)warp * R * STAGE;
    if (lane == 0) {
        for (int i = 0; i < R; ++i) mbar_init(full + i, 1);
        mbar_fence_init();
    }
    __syncwarp();

    // per-CTA arrival counters of the pairs its warps share (level 1 of the split-pair combine)
    __shared__ unsigned s_lcnt[kLocalPairs];
    __shared__ float s_ss[EPI ? kConsumers : 1][EPI ? kSsMax : 1];   // deferred-norm sums (QbInNorm), per warp
    __shared__ unsigned s_arrive;   // TP: warps of this CTA that are done
    for (int i = threadIdx.x; i < kLocalPairs; i += kThreads) s_lcnt[i] = 0u;
    if (threadIdx.x == 0) s_arrive = 0u;
    __syncthreads();
    const int gw = blockIdx.x * kConsumers + warp;
    if (gw >= p.Wt) {
        if (TP) {
            pdl_wait();   // arrive only after the previous TP launch has finished its own count
            tp_arrive(p.tp, smem_u32(&s_arrive), lane);
        }
        return;
    }
    const int grp_pair0 = warp_s0(p.S, p.Wt, (gw / p.group) * p.group) / p.nb;
    const int s0 = warp_s0(p.S, p.Wt, gw), s1 = warp_s0(p.S, p.Wt, gw + 1);
    const int n = s1 - s0;
    // producer cursor (lane 0): source of the next stage, its block, pairs left in the segment
    int ib, iseg = 0, seg_pairs_left;
    const uint8_t* src;
    {
        const int ip = s0 / p.nb;
        ib = s0 - ip * p.nb;
        while (iseg + 1 < p.nseg && ip >= p.pair0[iseg + 1]) ++iseg;
        src = p.seg[iseg].w + ((size_t)(ip - p.pair0[iseg]) * 2 * p.nb + ib) * TB;
        seg_pairs_left = p.pair0[iseg + 1] - ip;
    }
    const size_t tile_bytes = (size_t)p.nb * TB;   // the units of one tile
    const uint32_t ring_s = smem_u32(ring), full_s = smem_u32(full);
    auto issue = [&](int slot) {
        const uint32_t dst = ring_s + (uint32_t)slot * STAGE, bar = full_s + (uint32_t)slot * 8u;
        mbar_expect_tx_s(bar, STAGE);
        bulk_g2s_s(dst, src, TB, bar);
        bulk_g2s_s(dst + TB, src + tile_bytes, TB, bar);
        src += TB;
        if (++ib == p.nb) {
            ib = 0;
            src += tile_bytes;   // past the pair's second tile
            if (--seg_pairs_left == 0 && iseg + 1 < p.nseg) {
                ++iseg;
                src = p.seg[iseg].w;
                seg_pairs_left = p.pair0[iseg + 1] - p.pair0[iseg];
            }
        }
    };
    // weights do not depend on the previous kernel: start streaming before the wait
    if (lane == 0)
        for (int r = 0; r < R && r < n; ++r) issue(r);
    pdl_wait();   // activations written by the previous kernel are complete from here on
    // let the next launch start only now: triggered at entry, a chain of GEMVs had CTAs of
    // the next two launches resident and idle in their wait, crowding this one onto fewer SMs
    pdl_trigger();
    // the deferred norm's per-block sums: copied now, read at the first pair finish
    if (EPI && p.in_ss && p.N * p.nb <= kSsMax)
        for (int i = lane; i < p.N * p.nb; i += 32) cp_async4(&s_ss[warp][i], p.in_ss + i);

    float acc[2][NT][4];   // fp16 path: mma accumulator layout
    float tk[2][2][2];     // int8 path: (tile, row g + 8r, token c + 4k)
    auto reset = [&]() {
        zero<NT>(acc[0]);
        zero<NT>(acc[1]);
#pragma unroll
        for (int t = 0; t < 2; ++t) tk[t][0][0] = tk[t][0][1] = tk[t][1][0] = tk[t][1][1] = 0.f;
    };
    auto finish = [&](int pair) {
        float o[2][4];
        bool active;
        if (I8) pair_out_i8<NT>(tk, o, active, lane);
        else pair_out_f16<NT>(acc, o, active, lane);
        finish_pair<EPI, TP>(p, pair, gw, s0, s1, o, active, lane, s_lcnt, grp_pair0, s_ss[EPI ? warp : 0]);
    };
    reset();
    const int c = lane & 3;
    int cp = s0 / p.nb, cb = s0 - cp * p.nb;
    // int8 path: B fragments of sub-blocks 0, 1 of the next stage (prefetched one stage ahead)
    uint2 bpre[2][NT == 1 ? 2 : 3];
    if constexpr (I8) {
        constexpr int NTI = NT == 1 ? 2 : 3;
        load_bq<NTI>(bpre[0], p.xq + (size_t)cb * 8 * NTI * 32, 0, lane);
        load_bq<NTI>(bpre[1], p.xq + (size_t)cb * 8 * NTI * 32, 1, lane);
    }
    int cur_pair = cp;
    int slot = 0;
    uint32_t phase = 0;
    for (int r = 0; r < n; ++r) {
        if (cp != cur_pair) {
            finish(cur_pair);
            reset();
            cur_pair = cp;
        }
        if (!mbar_wait(full + slot, phase)) {
            // give up: record it, let the copies this warp issued land, return
            if (lane == 0) {
                atomicExch(p.err, 2u);
                int sl = slot;
                uint32_t ph = phase;
                for (int q = r; q < n && q < r + R; ++q) {
                    mbar_wait(full + sl, ph, 1u << 20);
                    if (++sl == R) { sl = 0; ph ^= 1u; }
                }
            }
            return;
        }
        const int b = cb;
        const uint8_t* u = ring + (size_t)slot * STAGE;
        if constexpr (I8) {
            constexpr int NTI = NT == 1 ? 2 : 3;
            float xs[NT];
#pragma unroll
            for (int k = 0; k < NT; ++k) {
                const int tok = c + 4 * k;
                xs[k] = tok < p.N ? __ldg(p.xqscale + tok * p.nb + b) : 0.f;
            }
            const int b_next = b + 1 == p.nb ? 0 : b + 1;
            float v[2][2][2];
            stage_iq4_i8<NTI>(u, p.xq + (size_t)b * 8 * NTI * 32, p.xq + (size_t)b_next * 8 * NTI * 32, lane,
                              bpre, v);
            __syncwarp();   // every lane is done with the slot
            if (lane == 0 && r + R < n) issue(slot);
            if (++slot == R) {
                slot = 0;
                phase ^= 1u;
            }
#pragma unroll
            for (int k = 0; k < NT; ++k)
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    tk[t][0][k] = fmaf(xs[k], v[t][0][k], tk[t][0][k]);
                    tk[t][1][k] = fmaf(xs[k], v[t][1][k], tk[t][1][k]);
                }
        } else {
            const uint2* xf = p.xfrag + (size_t)b * 16 * NT * 32;
            float ab[2][NT][4], mt[2][NT][4];
            zero<NT>(ab[0]);
            zero<NT>(ab[1]);
            zero<NT>(mt[0]);
            zero<NT>(mt[1]);
            if (FMT == QB_Q8_0) stage_q8_0<NT>(u, xf, lane, ab, mt);
            else if (FMT == QB_Q6_K) stage_q6k<NT>(u, xf, lane, ab, mt);
            else if (FMT == QB_Q4_K) stage_qk<NT, false>(u, xf, p.xsum + b * 8, p.K >> 5, lane, ab, mt);
            else if (FMT == QB_Q5_K) stage_qk<NT, true>(u, xf, p.xsum + b * 8, p.K >> 5, lane, ab, mt);
            __syncwarp();   // every lane is done with the slot
            if (lane == 0 && r + R < n) issue(slot);
            if (++slot == R) {
                slot = 0;
                phase ^= 1u;
            }
#pragma unroll
            for (int ct = 0; ct < NT; ++ct)
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float xs = __ldg(p.xscale + col_token<NT>(ct, 2 * c + i) * p.nb + b);
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        acc[t][ct][i] = fmaf(xs, ab[t][ct][i], acc[t][ct][i]) + mt[t][ct][i];
                        acc[t][ct][2 + i] = fmaf(xs, ab[t][ct][2 + i], acc[t][ct][2 + i]) + mt[t][ct][2 + i];
                    }
                }
        }
        if (++cb == p.nb) {
            cb = 0;
            ++cp;
        }
    }
    if (cur_pair >= 0) finish(cur_pair);
    if (TP) tp_arrive(p.tp, smem_u32(&s_arrive), lane);
}

// ----------------------- tensor-parallel reduction ------------------------
struct TpR {
    int world;
    const uint2* part[QB_TP_MAX];   // rank r's part buffer (2 slots of (value, tag)), mapped here
    long long slot;
    const unsigned* seq;
    unsigned* err;
};

// x += sum over ranks of the last partial-mode launch's partial sums, in rank
// order (every rank adds the same numbers in the same order).  A partial sum
// counts once its tag equals this rank's sequence number, which that launch
// advanced: an element not yet tagged is re-read (bounded).
__global__ void __launch_bounds__(256) tp_reduce_kernel(float* __restrict__ x, long long ldx, int E, int N, TpR r) {
    pdl_wait();
    pdl_trigger();
    const unsigned sq = *(volatile const unsigned*)r.seq;
    const size_t off = (size_t)((sq - 1u) & 1u) * r.slot;   // the slot the partial launch wrote
    const int n2 = E >> 1;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N * n2) return;
    const int t = i / n2, e = (i - t * n2) * 2;
    const size_t pe = off + (size_t)t * E + e;
    float a0 = 0.f, a1 = 0.f;
    for (int q = 0; q < r.world; ++q) {
        const uint4* src = reinterpret_cast<const uint4*>(r.part[q] + pe);
        uint4 v;
        const unsigned long long t0 = global_ns();
        for (uint32_t it = 0;; ++it) {
            asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(src) : "memory");
            if (v.y == sq && v.w == sq) break;
            if (peer_wait_over(it, t0, r.err, 4u)) return;
            __nanosleep(32);
        }
        if (q == 0) {
            a0 = __uint_as_float(v.x);
            a1 = __uint_as_float(v.z);
        } else {
            a0 += __uint_as_float(v.x);
            a1 += __uint_as_float(v.z);
        }
    }
    float2* xp = reinterpret_cast<float2*>(x + (size_t)t * ldx + e);
    float2 xv = *xp;
    xv.x += a0;
    xv.y += a1;
    *xp = xv;
}

// ------------------------------- F32 ---------------------------------------
// Plain fp32 rows (src/kernels.c:342-357).  One warp per row.
__global__ void qmv_f32_kernel(const float* __restrict__ W, int rows, int K, const float* __restrict__ x,
                               long long ldx, int N, float* __restrict__ out, long long ldo, int accumulate,
                               int row_lo, int row_hi) {
    pdl_wait();
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int r = row_lo + warp;
    if (r >= row_hi || r >= rows) return;
    const float* wr = W + (size_t)r * K;
    for (int t = 0; t < N; ++t) {
        float s = 0.f;
        for (int k = lane; k < K; k += 32) s = fmaf(wr[k], x[(size_t)t * ldx + k], s);
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
            float* dst = out + (size_t)t * ldo + r;
            *dst = accumulate ? (*dst + s) : s;
        }
    }
}

// ------------------------------- repack ------------------------------------
// One warp per (tile, unit).  src rows are GGUF rows of row_bytes bytes; rows
// beyond `rows` (padding to a whole tile pair) are written as zeros.

__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

__global__ void repack_kernel(int type, const uint8_t* __restrict__ src, size_t row_bytes, int rows,
                              int units_per_row, uint8_t* __restrict__ dst, long long n_units_total) {
    const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= n_units_total) return;
    const int tile = (int)(gw / units_per_row), u = (int)(gw % units_per_row);
    const int g = lane >> 2, c = lane & 3;
    const int UB = qb_unit_bytes(type);
    uint8_t* d = dst + (size_t)gw * UB;
    const int src_block = type == QB_Q8_0 ? 34 : type == QB_IQ4_XS ? 136 : UB / 16;
    auto rowp = [&](int rr) -> const uint8_t* {
        const int r = tile * QB_TILE + rr;
        return r < rows ? src + (size_t)r * row_bytes + (size_t)u * src_block : nullptr;
    };
    auto w32 = [&](const uint8_t* rp, int off) -> uint32_t { return rp ? ld_u32_unaligned(rp + off) : 0u; };
    const uint8_t* pg = rowp(g);
    const uint8_t* pg8 = rowp(g + 8);
    uint32_t* d32 = reinterpret_cast<uint32_t*>(d);

    if (type == QB_IQ4_XS) {
        for (int p = 0; p < 4; ++p) {
            d32[(p * 512 + lane * 16) / 4 + 0] = w32(pg, 8 + 16 * (2 * p) + 4 * c);
            d32[(p * 512 + lane * 16) / 4 + 1] = w32(pg8, 8 + 16 * (2 * p) + 4 * c);
            d32[(p * 512 + lane * 16) / 4 + 2] = w32(pg, 8 + 16 * (2 * p + 1) + 4 * c);
            d32[(p * 512 + lane * 16) / 4 + 3] = w32(pg8, 8 + 16 * (2 * p + 1) + 4 * c);
        }
        if (lane < 16) {
            // ls_ib = scales_l nibble ib | scales_h bits 2ib..2ib+1 << 4 (src/kernels.c:84-90),
            // stored as the differences ls_j - ls_{j+1} (j < 7) and ls_7 - 32
            const uint8_t* rp = rowp(lane);
            uint32_t D0 = 0, D1 = 0, dd = 0;
            if (rp) {
                const uint32_t sh = rp[2] | (rp[3] << 8);
                const uint32_t sl = w32(rp, 4);
                int ls[9];
                for (int ib = 0; ib < 8; ++ib) ls[ib] = (int)(((sl >> (4 * ib)) & 0xF) | (((sh >> (2 * ib)) & 3) << 4));
                ls[8] = 32;
                for (int j = 0; j < 4; ++j) {
                    D0 |= ((uint32_t)(ls[j] - ls[j + 1]) & 0xFFu) << (8 * j);
                    D1 |= ((uint32_t)(ls[4 + j] - ls[5 + j]) & 0xFFu) << (8 * j);
                }
                dd = rp[0] | (rp[1] << 8);
            }
            d32[(kIq4Dl + lane * 8) / 4 + 0] = D0;
            d32[(kIq4Dl + lane * 8) / 4 + 1] = D1;
            reinterpret_cast<uint16_t*>(d + kIq4D)[lane] = (uint16_t)dd;
        }
    } else if (type == QB_Q8_0) {
        d32[lane * 4 + 0] = w32(pg, 2 + 4 * c);
        d32[lane * 4 + 1] = w32(pg8, 2 + 4 * c);
        d32[lane * 4 + 2] = w32(pg, 2 + 16 + 4 * c);
        d32[lane * 4 + 3] = w32(pg8, 2 + 16 + 4 * c);
        if (lane < 16) {
            const uint8_t* rp = rowp(lane);
            reinterpret_cast<uint16_t*>(d + 512)[lane] = rp ? (uint16_t)(rp[0] | (rp[1] << 8)) : 0;
        }
    } else if (type == QB_Q4_K || type == QB_Q5_K) {
        const int qs_off = type == QB_Q5_K ? 48 : 16;
        for (int j = 0; j < 4; ++j) {
            d32[(j * 512 + lane * 16) / 4 + 0] = w32(pg, qs_off + 32 * j + 4 * c);
            d32[(j * 512 + lane * 16) / 4 + 1] = w32(pg, qs_off + 32 * j + 16 + 4 * c);
            d32[(j * 512 + lane * 16) / 4 + 2] = w32(pg8, qs_off + 32 * j + 4 * c);
            d32[(j * 512 + lane * 16) / 4 + 3] = w32(pg8, qs_off + 32 * j + 16 + 4 * c);
        }
        int hdr = 2048;
        if (type == QB_Q5_K) {
            d32[(2048 + lane * 16) / 4 + 0] = w32(pg, 16 + 4 * c);
            d32[(2048 + lane * 16) / 4 + 1] = w32(pg, 16 + 16 + 4 * c);
            d32[(2048 + lane * 16) / 4 + 2] = w32(pg8, 16 + 4 * c);
            d32[(2048 + lane * 16) / 4 + 3] = w32(pg8, 16 + 16 + 4 * c);
            hdr = 2560;
        }
        if (lane < 16) {
            const uint8_t* rp = rowp(lane);
            for (int i = 0; i < 4; ++i) d32[(hdr + lane * 16) / 4 + i] = w32(rp, 4 * i);
        }
    } else if (type == QB_Q6_K) {
        // ql[128] qh[64] scales[16] d(2).  Element e of group G (16G + l'):
        // n = G/8, m = (G%8)/2, is = G%2, l = 16is + l'
        // q = (ql[64n + 32(m&1) + l] >> 4(m>>1)) & 15 | ((qh[32n + l] >> 2m) & 3) << 4
        auto q6 = [&](const uint8_t* rp, int e) -> uint32_t {
            if (!rp) return 0u;
            const int G = e >> 4, lp = e & 15;
            const int n = G >> 3, m = (G & 7) >> 1, is = G & 1, l = 16 * is + lp;
            const uint32_t lo = (rp[64 * n + 32 * (m & 1) + l] >> (4 * (m >> 1))) & 15u;
            const uint32_t hi = (rp[128 + 32 * n + l] >> (2 * m)) & 3u;
            return lo | (hi << 4);
        };
        for (int qc = 0; qc < 4; ++qc)
            for (int i = 0; i < 4; ++i) {
                const int G = 4 * qc + i;
                uint32_t wv = 0;
                for (int k = 0; k < 4; ++k) {
                    wv |= (q6(pg, 16 * G + 4 * c + k) & 15u) << (4 * k);
                    wv |= (q6(pg8, 16 * G + 4 * c + k) & 15u) << (16 + 4 * k);
                }
                d32[(qc * 512 + lane * 16) / 4 + i] = wv;
            }
        for (int mp = 0; mp < 8; ++mp) {
            uint32_t wv = 0;
            for (int j = 0; j < 4; ++j) {
                const uint8_t* rp = j < 2 ? pg : pg8;
                const int ee = (j & 1) ? 2 : 0;
                for (int half = 0; half < 2; ++half) {
                    const int G = 2 * mp + half;
                    const uint32_t ev = q6(rp, 16 * G + 4 * c + ee) >> 4;
                    const uint32_t od = q6(rp, 16 * G + 4 * c + ee + 1) >> 4;
                    const int sh = half == 0 ? 4 : 0;
                    wv |= ((ev & 3u) << (8 * j + sh)) | ((od & 3u) << (8 * j + sh + 2));
                }
            }
            d32[(2048 + (mp >> 2) * 512 + lane * 16) / 4 + (mp & 3)] = wv;
        }
        if (lane < 16) {
            const uint8_t* rp = rowp(lane);
            // int8 scales stored as sc + 128 (unsigned): one byte permute makes the float 2^23 + sc + 128
            for (int i = 0; i < 4; ++i) d32[(3072 + lane * 16) / 4 + i] = w32(rp, 192 + 4 * i) ^ 0x80808080u;
            reinterpret_cast<uint16_t*>(d + 3328)[lane] = rp ? (uint16_t)(rp[208] | (rp[209] << 8)) : 0;
        }
    }
}

// ------------------------- activation fragments ------------------------------
// x [N][ldx] fp32 -> xfrag (hi/lo fp16, B-fragment order), xscale, xsum.
// Optional RMSNorm folded in: y = (x * inv_rms) * w  (src/kernels.c:741-777);
// every CTA computes its token's inv_rms itself (the row is a few KB), so the
// grid spreads over all 256-column blocks.  Two segments allow the MTP concat
// [RMSNorm(e, enorm) || RMSNorm(h, hnorm)] (src/model.c:1044-1047).

struct XSeg {
    const float* x;
    long long ldx;
    const float* w;
    int len;
};

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += sh[i];
    return s;
}

__global__ void __launch_bounds__(256) xprep_kernel(XSeg s0, XSeg s1, int nseg, int N, float eps, QbXBuf xb,
                                                    int what) {
    // a GEMV follows: release it before waiting, so that its CTAs take their places and
    // start streaming weights while this short kernel runs
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    const int K = s0.len + (nseg > 1 ? s1.len : 0);
    const int nb = K >> 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __shared__ float sh[32];
    // this warp's block: its loads go out before the row reductions (one round trip, not two)
    const int b = blockIdx.x * nw + warp;
    const bool has_block = b < nb;
    const int col0 = b * 256;
    const int si = (nseg > 1 && col0 >= s0.len) ? 1 : 0;
    const XSeg& S = si ? s1 : s0;
    const int lc0 = col0 - (si ? s0.len : 0);
    float v[8], wv[8];
    if (has_block) {
        const float* x = S.x + (size_t)t * S.ldx + lc0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float4 xv = *reinterpret_cast<const float4*>(x + h * 128 + 4 * lane);
            v[4 * h + 0] = xv.x; v[4 * h + 1] = xv.y; v[4 * h + 2] = xv.z; v[4 * h + 3] = xv.w;
            if (S.w) {
                const float4 w4 = *reinterpret_cast<const float4*>(S.w + lc0 + h * 128 + 4 * lane);
                wv[4 * h + 0] = w4.x; wv[4 * h + 1] = w4.y; wv[4 * h + 2] = w4.z; wv[4 * h + 3] = w4.w;
            }
        }
    }
    float inv[2] = {1.f, 1.f};
    for (int sj = 0; sj < nseg; ++sj) {
        const XSeg& Q = sj ? s1 : s0;
        if (!Q.w) continue;
        const float* x = Q.x + (size_t)t * Q.ldx;
        float ss = 0.f;
        for (int i = threadIdx.x * 4; i < Q.len; i += blockDim.x * 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(x + i);
            ss = fmaf(q4.x, q4.x, ss);
            ss = fmaf(q4.y, q4.y, ss);
            ss = fmaf(q4.z, q4.z, ss);
            ss = fmaf(q4.w, q4.w, ss);
        }
        ss = block_sum(ss, sh);
        inv[sj] = 1.0f / sqrtf(ss / (float)Q.len + eps);
    }
    if (!has_block) return;
    if (S.w) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (v[i] * inv[si]) * wv[i];
    }
    xprep_emit(v, t, b, N, nb, K, xb, what, lane);
}

}  // namespace

// ============================ host launchers ==================================

// repacked matrices are padded to whole 32-row tile pairs
static size_t padded_tiles(int rows) { return (size_t)((rows + 31) / 32) * 2; }

size_t qb_repacked_bytes(int type, int rows, int K) {
    const int ub = qb_unit_bytes(type), uc = qb_unit_cols(type);
    if (!ub || K % 256) return 0;
    return padded_tiles(rows) * (size_t)(K / uc) * ub;
}

cudaError_t qb_repack(int type, const void* src_dev, int rows, int K, void* dst_dev, cudaStream_t st) {
    const int ub = qb_unit_bytes(type), uc = qb_unit_cols(type);
    if (!ub || K % 256) return cudaErrorInvalidValue;
    const int upr = K / uc;
    const size_t row_bytes = (size_t)upr * (type == QB_Q8_0 ? 34 : type == QB_IQ4_XS ? 136 : ub / 16);
    const long long units = (long long)padded_tiles(rows) * upr;
    const int threads = 256;
    const long long blocks = (units * 32 + threads - 1) / threads;
    repack_kernel<<<(unsigned)blocks, threads, 0, st>>>(type, (const uint8_t*)src_dev, row_bytes, rows, upr,
                                                        (uint8_t*)dst_dev, units);
    return cudaGetLastError();
}

size_t qb_xfrag_bytes(int K) { return (size_t)(K + 255) / 256 * 256 / 16 * 2 * 32 * sizeof(uint2); }
size_t qb_xq_bytes(int K) { return (size_t)(K + 255) / 256 * 256 / 32 * 3 * 32 * sizeof(uint2); }

size_t qb_xtc_bytes(int K) { return (size_t)(K + 255) / 256 * 4096; }
size_t qb_xtc16_bytes(int K) { return (size_t)(K + 255) / 256 * 12288; }
size_t qb_xtc32_bytes(int K) { return (size_t)(K + 255) / 256 * 24576; }

int qb_xprep_needs(int type, int N, int tc) {
    switch (type) {
    case QB_IQ4_XS: return (tc && N <= 4) ? QB_XP_TC : QB_XP_I8;
    case QB_Q4_K:
    case QB_Q5_K: return QB_XP_F16 | QB_XP_SUM;
    case QB_Q6_K:
    case QB_Q8_0: return QB_XP_F16;
    default: return 0;
    }
}

cudaError_t qb_xprep(const QbXIn* in, int nseg, int N, float eps, const QbXBuf& xb, int what, cudaStream_t st) {
    XSeg s[2] = {};
    int K = 0;
    // up to QB_MAX_TOK tokens; or up to QB_WIDE, the 8-row formats in chunks of
    // QB_MAX_TOK rows (QbXBuf chunk strides set), the 16-token tiles up to 16 rows
    if (nseg < 1 || nseg > 2 || N < 1 || N > QB_WIDE) return cudaErrorInvalidValue;
    if (N > QB_MAX_TOK && ((what & QB_XP_TC) || ((what & QB_XP_TC16) && N > QB_TC16_TOK) ||
                           ((what & QB_XP_F16) && !xb.cs_frag) || ((what & QB_XP_I8) && !xb.cs_q)))
        return cudaErrorInvalidValue;
    for (int i = 0; i < nseg; ++i) {
        s[i].x = in[i].x;
        s[i].ldx = in[i].ldx;
        s[i].w = in[i].norm_w;
        s[i].len = in[i].len;
        if (in[i].len % 256) return cudaErrorInvalidValue;
        K += in[i].len;
    }
    if (((what & QB_XP_F16) && (!xb.xfrag || !xb.xscale)) || ((what & QB_XP_SUM) && !xb.xsum) ||
        ((what & QB_XP_I8) && (!xb.xq || !xb.xqscale)) || ((what & QB_XP_TC) && (!xb.xtc || !xb.xqscale || N > 4)) ||
        ((what & QB_XP_TC16) && (!xb.xtc16 || !xb.xqscale)) || ((what & QB_XP_TC32) && (!xb.xtc32 || !xb.xqscale)))
        return cudaErrorInvalidValue;
    const int nb = K / 256;
    return qb_launch(xprep_kernel, dim3((nb + 7) / 8, N), dim3(256), 0, st, s[0], s[1], nseg, N, eps, xb, what);
}

static int g_num_sms = 0;

namespace {
cudaError_t qmv_launch(int type, const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate,
                       int row_lo, int row_hi, const QbInNorm* in_norm, const QbEpi* epi, const QbTp* tp,
                       const QbQmvWork& work, cudaStream_t st) {
    const bool tp_k = tp && tp->world > 1;
    if (nseg < (tp_k ? 0 : 1) || nseg > QB_MAX_SEG || N < 1 || N > QB_MAX_TOK || K % 256) return cudaErrorInvalidValue;
    if (tp_k && (tp->world > QB_TP_MAX || tp->rank < 0 || tp->rank >= tp->world || !tp->flags || !tp->done || !tp->seq ||
                 (epi && epi->kind != QB_EPI_NONE) || (in_norm && in_norm->ss)))
        return cudaErrorInvalidValue;
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    QmvK p = {};
    int pairs = 0;
    for (int i = 0; i < nseg; ++i) {
        p.seg[i].w = (const uint8_t*)segs[i].w;
        p.seg[i].out = segs[i].out;
        p.seg[i].ldo = segs[i].ldo;
        p.seg[i].rows = segs[i].rows;
        p.pair0[i] = pairs;
        pairs += (segs[i].rows + 31) / 32;
    }
    p.pair0[nseg] = pairs;
    if (pairs > work.max_pairs) return cudaErrorInvalidValue;
    p.nseg = nseg;
    p.K = K;
    p.nb = K / 256;
    p.N = N;
    const long long S64 = (long long)pairs * p.nb;
    if (S64 * (long long)work.max_warps >= (1ll << 31)) return cudaErrorInvalidValue;
    p.S = (int)S64;
    const int tb = tile_block_bytes(type);
    if (!tb) return cudaErrorInvalidValue;
    const int stage = 2 * tb;
    int R = (kSmemBudget - kRingOff) / (kConsumers * stage);
    if (R > 8) R = 8;
    if (R < 2) R = 2;
    p.stages_per_warp_ring = R;
    const size_t smem = kRingOff + (size_t)kConsumers * R * stage;
    // every warp owns >= 1 stage (Wt <= S); aim for >= QB_QMV_MIN_STAGES stages per warp
    int grid = g_num_sms * kCtasPerSm;
    const int warps_needed = (p.S + kMinStagesPerWarp - 1) / kMinStagesPerWarp;
    if (grid * kConsumers > warps_needed) grid = (warps_needed + kConsumers - 1) / kConsumers;
    if (grid < 1) grid = 1;
    while (grid > 1 && grid * kConsumers > p.S) --grid;
    p.Wt = grid * kConsumers < p.S ? grid * kConsumers : p.S;   // warps beyond Wt exit at once (S == 0: all)
    if (p.Wt > work.max_warps) return cudaErrorInvalidValue;
    p.xfrag = xb.xfrag;
    p.xscale = xb.xscale;
    p.xsum = xb.xsum;
    p.xq = xb.xq;
    p.xqscale = xb.xqscale;
    const int need = qb_xprep_needs(type, N, 0);
    if (((need & QB_XP_F16) && (!p.xfrag || !p.xscale)) || ((need & QB_XP_SUM) && !p.xsum) ||
        ((need & QB_XP_I8) && (!p.xq || !p.xqscale)))
        return cudaErrorInvalidValue;
    p.accumulate = accumulate;
    p.row_lo = row_lo;
    p.row_hi = row_hi;
    p.partial = work.partial;
    p.gpartial = work.gpartial;
    p.counters = work.counters;
    if (p.Wt > 0) {   // CTA-level combine when a CTA's stage range touches at most kLocalPairs pairs
        const long long per_cta = ((long long)p.S * kConsumers + p.Wt - 1) / p.Wt;   // stages of 8 warps
        p.group = per_cta / p.nb + 2 <= kLocalPairs ? kConsumers : 1;
    } else {
        p.group = 1;
    }
    if (tp_k) {
        p.tp.np = tp->world - 1;
        p.tp.rank = tp->rank;
        for (int i = 0; i < tp->world - 1; ++i) p.tp.delta[i] = tp->delta[i];
        p.tp.flags = tp->flags;
        p.tp.done = tp->done;
        p.tp.seq = tp->seq;
        p.tp.err = work.err;
        p.tp.gather = tp->gather;
        p.tp.part = reinterpret_cast<uint2*>(tp->part);
        p.tp.part_slot = tp->part_slot;
        if (!tp->gather && (!tp->part || accumulate || nseg > 1 || (nseg == 1 && segs[0].ldo * QB_MAX_TOK > tp->part_slot)))
            return cudaErrorInvalidValue;
    }
    p.err = work.err;
    if (in_norm && in_norm->ss) {
        p.in_ss = in_norm->ss;
        p.in_eps = in_norm->eps;
    }
    if (epi && epi->kind != QB_EPI_NONE) {
        // one matrix, whole output, whole 256-row blocks; the fragments go to another buffer
        const int rows = segs[0].rows;
        const bool swiglu = epi->kind == QB_EPI_SWIGLU;
        const int next_k = swiglu ? rows / 2 : rows;
        if (nseg != 1 || row_lo > 0 || row_hi < rows || next_k % 256 || !work.bcounters ||
            (epi->kind != QB_EPI_NORM && !swiglu) || (swiglu && (accumulate || !epi->h || epi->ldh < next_k)) ||
            (!swiglu && (!epi->norm_w || !epi->ss)) || epi->xb.xq == xb.xq || epi->xb.xfrag == xb.xfrag ||
            next_k / 256 > work.max_pairs)
            return cudaErrorInvalidValue;
        const int what = epi->what;
        if (((what & QB_XP_F16) && (!epi->xb.xfrag || !epi->xb.xscale)) || ((what & QB_XP_SUM) && !epi->xb.xsum) ||
            ((what & QB_XP_I8) && (!epi->xb.xq || !epi->xb.xqscale)) || (what & QB_XP_TC) || !what)
            return cudaErrorInvalidValue;
        p.epi = epi->kind;
        p.bcnt = work.bcounters;
        p.epi_w = epi->norm_w;
        p.epi_ss = epi->ss;
        p.epi_h = epi->h;
        p.epi_ldh = epi->ldh;
        p.epi_K = next_k;
        p.epi_what = what;
        p.epi_xb = epi->xb;
    }
    const bool nt2 = N > 4;
    const bool epi_k = p.in_ss != nullptr || p.epi != QB_EPI_NONE;
    // a grid of at most one CTA per SM asks for more than half of an SM's shared memory:
    // CTAs placed early, while the previous kernels still hold SMs, then cannot pair up on
    // the SMs that free first
    const size_t smem_launch = grid <= g_num_sms && smem < (size_t)116 * 1024 ? (size_t)116 * 1024 : smem;
    cudaError_t e = cudaSuccess;
#define QB_LAUNCH(F, I8)                                                                               \
    do {                                                                                               \
        auto kern = tp_k    ? (nt2 ? qmv_kernel<F, 2, I8, false, true> : qmv_kernel<F, 1, I8, false, true>)   \
                    : epi_k ? (nt2 ? qmv_kernel<F, 2, I8, true, false> : qmv_kernel<F, 1, I8, true, false>)   \
                            : (nt2 ? qmv_kernel<F, 2, I8, false, false> : qmv_kernel<F, 1, I8, false, false>); \
        const int variant = nt2 + 2 * (epi_k ? 1 : tp_k ? 2 : 0);                                      \
        static bool attr_set[6] = {false, false, false, false, false, false};                          \
        if (!attr_set[variant]) {                                                                      \
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);       \
            attr_set[variant] = true;                                                                  \
        }                                                                                              \
        e = qb_launch(kern, dim3(grid), dim3(kThreads), smem_launch, st, p);                           \
    } while (0)
    switch (type) {
    case QB_IQ4_XS: QB_LAUNCH(QB_IQ4_XS, true); break;
    case QB_Q8_0: QB_LAUNCH(QB_Q8_0, false); break;
    case QB_Q4_K: QB_LAUNCH(QB_Q4_K, false); break;
    case QB_Q5_K: QB_LAUNCH(QB_Q5_K, false); break;
    case QB_Q6_K: QB_LAUNCH(QB_Q6_K, false); break;
    default: return cudaErrorInvalidValue;
    }
#undef QB_LAUNCH
    return e;
}
}  // namespace

cudaError_t qb_qmv(int type, const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate,
                   int row_lo, int row_hi, const QbQmvWork& work, cudaStream_t st) {
    return qmv_launch(type, segs, nseg, K, N, xb, accumulate, row_lo, row_hi, nullptr, nullptr, nullptr, work, st);
}

cudaError_t qb_qmv_ex(int type, const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate,
                      const QbInNorm* in_norm, const QbEpi* epi, const QbTp* tp, const QbQmvWork& work,
                      cudaStream_t st) {
    return qmv_launch(type, segs, nseg, K, N, xb, accumulate, 0, 1 << 30, in_norm, epi, tp, work, st);
}

cudaError_t qb_tp_reduce(float* x, long long ldx, int E, int N, const QbTp& tp, const void* const* parts,
                         unsigned* err, cudaStream_t st) {
    if (tp.world < 2 || tp.world > QB_TP_MAX || E % 4 || ldx % 2 || N < 1 || N > QB_MAX_TOK || !tp.seq)
        return cudaErrorInvalidValue;
    TpR r = {};
    r.world = tp.world;
    for (int q = 0; q < tp.world; ++q) {
        if (!parts[q]) return cudaErrorInvalidValue;
        r.part[q] = reinterpret_cast<const uint2*>(parts[q]);
    }
    r.slot = tp.part_slot;
    r.seq = tp.seq;
    r.err = err;
    const int n = N * (E / 2);
    return qb_launch(tp_reduce_kernel, dim3((n + 255) / 256), dim3(256), 0, st, x, ldx, E, N, r);
}

cudaError_t qb_interleave_tiles(int type, const void* a, const void* b, int rows, int K, void* dst, cudaStream_t st) {
    const int ub = qb_unit_bytes(type), uc = qb_unit_cols(type);
    if (!ub || K % 256 || rows % 16 || rows <= 0) return cudaErrorInvalidValue;
    const size_t tile = (size_t)(K / uc) * ub;   // the units of one 16-row tile
    const size_t tiles = (size_t)rows / 16;
    cudaError_t e = cudaMemcpy2DAsync(dst, 2 * tile, a, tile, tile, tiles, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return e;
    return cudaMemcpy2DAsync((uint8_t*)dst + tile, 2 * tile, b, tile, tile, tiles, cudaMemcpyDeviceToDevice, st);
}

cudaError_t qb_qmv_work_alloc(QbQmvWork& w, int max_pairs) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    w.max_warps = sms * kCtasPerSm * kConsumers;
    w.max_pairs = max_pairs;
    cudaError_t e;
    if ((e = cudaMalloc(&w.partial, (size_t)w.max_warps * 2 * 256 * sizeof(float))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&w.gpartial, (size_t)w.max_warps * 2 * 256 * sizeof(float))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&w.counters, (size_t)max_pairs * sizeof(unsigned))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&w.bcounters, (size_t)max_pairs * sizeof(unsigned))) != cudaSuccess) return e;
    if ((e = cudaMemset(w.bcounters, 0, (size_t)max_pairs * sizeof(unsigned))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&w.err, sizeof(unsigned))) != cudaSuccess) return e;
    if ((e = cudaMemset(w.counters, 0, (size_t)max_pairs * sizeof(unsigned))) != cudaSuccess) return e;
    w.max_tc_ctas = qb_qmv_tc_max_ctas();
    w.max_tc_rows = (long long)max_pairs * 32 + 128 * QB_MAX_SEG;   // every fused matrix rounds up to a tile
    if ((e = cudaMalloc(&w.tc_partial, qb_qmv_tc_partial_floats(w.max_tc_ctas) * sizeof(float))) != cudaSuccess)
        return e;
    // per row (qb_qmv_tc), or per row and token group of 8 (qb_qmv_tcw)
    if ((e = cudaMalloc(&w.tc_counters, (size_t)w.max_tc_rows * 4 * sizeof(unsigned))) != cudaSuccess) return e;
    if ((e = cudaMemset(w.tc_counters, 0, (size_t)w.max_tc_rows * 4 * sizeof(unsigned))) != cudaSuccess) return e;
    if ((e = cudaMemset(w.err, 0, sizeof(unsigned))) != cudaSuccess) return e;
    return cudaDeviceSynchronize();
}

void qb_qmv_work_free(QbQmvWork& w) {
    if (w.partial) cudaFree(w.partial);
    if (w.gpartial) cudaFree(w.gpartial);
    if (w.tc_partial) cudaFree(w.tc_partial);
    if (w.tc_counters) cudaFree(w.tc_counters);
    if (w.counters) cudaFree(w.counters);
    if (w.bcounters) cudaFree(w.bcounters);
    if (w.err) cudaFree(w.err);
    w = QbQmvWork{};
}

cudaError_t qb_qmv_f32(const float* W, int rows, int K, const float* x, long long ldx, int N, float* out,
                       long long ldo, int accumulate, int row_lo, int row_hi, cudaStream_t st) {
    const int n = row_hi - row_lo;
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    const int blocks = (n * 32 + threads - 1) / threads;
    return qb_launch(qmv_f32_kernel, dim3(blocks), dim3(threads), 0, st, W, rows, K, x, ldx, N, out, ldo, accumulate,
                     row_lo, row_hi);
}
