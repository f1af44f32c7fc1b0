// Quantised GEMV on the sm_100a tensor cores: out[t][r] = sum_k W[r][k] * x[t][k]
// for up to 8 input vectors, weights streamed once from HBM.
//
// Reference: dot_*_b / gemv_rows_batch / gemv_multi_batch, src/kernels.c:323-736
// (one weight sweep serves all n <= GEMV_MAX_B vectors).  The block formats
// and their dequantisation are those of include/quant.h:14-62 and
// src/quant.c:86-182.
//
// Design.  The weights are repacked once at load time from GGUF super-blocks
// into 16-row tiles whose bytes land directly in mma.sync m16n8k16 A-fragment
// order (same byte count, only reordered).  Inside the kernel each 4-bit /
// 6-bit / 8-bit code is expanded to an *exact* fp16 integer (IQ4 lookup table
// via byte permutes, K-quant codes via the 1024+q exponent trick), so the
// tensor core multiplies exact weight codes with the activations.  The
// activations are split into fp16 hi + lo halves (after a power-of-two scale
// per 256-column block), which keeps ~22 significant bits: the products are
// exact in the fp32 accumulator and the result carries fp32-level error.  The
// per-32 (IQ4_XS, Q4_K, Q5_K, Q8_0) or per-16 (Q6_K) block scales are
// applied to the fp32 partial sums after each sub-block's MMAs.
//
// mma k-index <-> element mapping, shared by every format and by the
// activation fragments: within the 16-element step s of a 32-element
// sub-block, thread c of a quad holds elements 16s+4c .. 16s+4c+3;
// (4c, 4c+1) form register 0/1 (k = 2c, 2c+1) and (4c+2, 4c+3) register 2/3
// (k = 2c+8, 2c+9).
#include "qb_common.cuh"
#include "qb_kernels.h"

namespace {

constexpr uint32_t H1152x2 = 0x64806480u;   // half2(1152, 1152) = 1024 + 128
constexpr uint32_t H1024x2 = 0x64006400u;   // half2(1024, 1024)
constexpr uint32_t H1056x2 = 0x64206420u;   // half2(1056, 1056) = 1024 + 32
constexpr uint32_t C64 = 0x64646464u;

// IQ4_NL table biased by +128 (reference src/quant.c:30-32: kvalues_iq4nl).
// u[v] = kvalues[v] + 128, packed four bytes per word, little endian.
__constant__ uint32_t c_iq4_lut[4];

// Expand 8 IQ4 nibbles (word = 4 qs bytes) into the four fp16x2 operands
// of the two k16 steps: out[0] = step0 reg(k 2c,2c+1), out[1] = step0 reg
// (k 2c+8,2c+9), out[2] / out[3] = step1.  Values are exact kvalues.
__device__ __forceinline__ void iq4_expand(uint32_t w, uint32_t T0, uint32_t T1, uint32_t T2,
                                           uint32_t T3, uint32_t (&o)[4]) {
    const uint32_t lo3 = w & 0x77777777u;
    const uint32_t sel = ((w >> 1) & 0x44444444u) | 0x32103210u;
    const uint32_t lo3h = lo3 >> 16;
    const uint32_t a = prmt(T0, T1, lo3), b = prmt(T2, T3, lo3);
    const uint32_t r_lo = prmt(a, b, sel);                 // [b0lo b0hi b1lo b1hi]
    const uint32_t ah = prmt(T0, T1, lo3h), bh = prmt(T2, T3, lo3h);
    const uint32_t r_hi = prmt(ah, bh, sel >> 16);         // [b2lo b2hi b3lo b3hi]
    o[0] = hsub2_u32(prmt(r_lo, C64, 0x5240u), H1152x2);   // elems 4c, 4c+1   (lo nibbles)
    o[1] = hsub2_u32(prmt(r_hi, C64, 0x5240u), H1152x2);   // elems 4c+2, 4c+3
    o[2] = hsub2_u32(prmt(r_lo, C64, 0x5341u), H1152x2);   // elems 16+4c, +1  (hi nibbles)
    o[3] = hsub2_u32(prmt(r_hi, C64, 0x5341u), H1152x2);
}

// 4 unsigned bytes (each < 256 after bias) -> two half2 (b0,b1), (b2,b3) = 1024 + byte
__device__ __forceinline__ void bytes_to_h2(uint32_t u, uint32_t& h01, uint32_t& h23) {
    h01 = prmt(u, C64, 0x5140u);
    h23 = prmt(u, C64, 0x7362u);
}

template <int NT>
__device__ __forceinline__ void mma_step(float (&cs)[NT][4], const uint32_t (&a)[4],
                                         const uint2* __restrict__ xf, int lane) {
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) {
        const uint2 b = __ldg(xf + ct * 32 + lane);
        mma_16816(cs[ct], a, b.x, b.y);
    }
}

template <int NT>
__device__ __forceinline__ void scale_acc(float (&ab)[NT][4], const float (&cs)[NT][4], float dg,
                                          float dg8) {
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) {
        ab[ct][0] = fmaf(dg, cs[ct][0], ab[ct][0]);
        ab[ct][1] = fmaf(dg, cs[ct][1], ab[ct][1]);
        ab[ct][2] = fmaf(dg8, cs[ct][2], ab[ct][2]);
        ab[ct][3] = fmaf(dg8, cs[ct][3], ab[ct][3]);
    }
}

// token index of accumulator column (ct, 2c+i)
template <int NT>
__device__ __forceinline__ int col_token(int ct, int col) {
    return NT == 1 ? (col & 3) : col;
}

// ---------------------------------------------------------------------------
// Per-format processing of one 256-column super-block for one 16-row tile.
// ab accumulates sum over sub-blocks of (block scale * tensor-core partial);
// xsum-based corrections (Q4_K/Q5_K mins) are returned in ab as well.

template <int NT>
__device__ __forceinline__ void blk_iq4xs(const uint8_t* __restrict__ unit, const uint2* __restrict__ xf,
                                          int lane, float (&ab)[NT][4]) {
    const int g = lane >> 2;
    const uint4 q0 = ldg_nc_128(unit + 0 * 512 + lane * 16);
    const uint4 q1 = ldg_nc_128(unit + 1 * 512 + lane * 16);
    const uint4 q2 = ldg_nc_128(unit + 2 * 512 + lane * 16);
    const uint4 q3 = ldg_nc_128(unit + 3 * 512 + lane * 16);
    const uint2 sg = ldg_nc_64(unit + 2048 + g * 8);
    const uint2 sg8 = ldg_nc_64(unit + 2048 + (g + 8) * 8);
    const float dg = h2f_bits(sg.x), dg8 = h2f_bits(sg8.x);
    const uint32_t shg = sg.x >> 16, shg8 = sg8.x >> 16;
    const uint32_t T0 = c_iq4_lut[0], T1 = c_iq4_lut[1], T2 = c_iq4_lut[2], T3 = c_iq4_lut[3];
    const uint4 qq[4] = {q0, q1, q2, q3};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int sb = 2 * p + h;
            const uint32_t wg = h ? qq[p].z : qq[p].x;
            const uint32_t wg8 = h ? qq[p].w : qq[p].y;
            uint32_t eg[4], eg8[4];
            iq4_expand(wg, T0, T1, T2, T3, eg);
            iq4_expand(wg8, T0, T1, T2, T3, eg8);
            float cs[NT][4];
#pragma unroll
            for (int ct = 0; ct < NT; ++ct) cs[ct][0] = cs[ct][1] = cs[ct][2] = cs[ct][3] = 0.f;
            {
                const uint32_t a[4] = {eg[0], eg8[0], eg[1], eg8[1]};
                mma_step<NT>(cs, a, xf + (sb * 2 + 0) * NT * 32, lane);
            }
            {
                const uint32_t a[4] = {eg[2], eg8[2], eg[3], eg8[3]};
                mma_step<NT>(cs, a, xf + (sb * 2 + 1) * NT * 32, lane);
            }
            // ls = 6-bit sub-block scale (src/kernels.c:84-90)
            const uint32_t lsg = ((sg.y >> (4 * sb)) & 0xFu) | (((shg >> (2 * sb)) & 3u) << 4);
            const uint32_t lsg8 = ((sg8.y >> (4 * sb)) & 0xFu) | (((shg8 >> (2 * sb)) & 3u) << 4);
            const float dlg = dg * (small_u2f(lsg) - 32.f);
            const float dlg8 = dg8 * (small_u2f(lsg8) - 32.f);
            scale_acc<NT>(ab, cs, dlg, dlg8);
        }
    }
}

template <int NT>
__device__ __forceinline__ void blk_q8_0(const uint8_t* __restrict__ unit0, const uint2* __restrict__ xf,
                                         int lane, float (&ab)[NT][4]) {
    const int g = lane >> 2;
#pragma unroll 2
    for (int sb = 0; sb < 8; ++sb) {
        const uint8_t* unit = unit0 + sb * 544;
        const uint4 q = ldg_nc_128(unit + lane * 16);
        const uint32_t dd = __ldg(reinterpret_cast<const unsigned short*>(unit + 512) + g) |
                            ((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(unit + 512) + g + 8) << 16);
        const float dg = h2f_bits(dd), dg8 = h2f_bits(dd >> 16);
        float cs[NT][4];
#pragma unroll
        for (int ct = 0; ct < NT; ++ct) cs[ct][0] = cs[ct][1] = cs[ct][2] = cs[ct][3] = 0.f;
        // words: [row g s0][row g8 s0][row g s1][row g8 s1]
        const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                               q.w ^ 0x80808080u};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            uint32_t a[4];
            bytes_to_h2(w[2 * s], a[0], a[2]);
            bytes_to_h2(w[2 * s + 1], a[1], a[3]);
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = hsub2_u32(a[i], H1152x2);
            mma_step<NT>(cs, a, xf + ((sb) * 2 + s) * NT * 32, lane);
        }
        scale_acc<NT>(ab, cs, dg, dg8);
    }
}

// Q4_K / Q5_K: w = d*sc*q - dmin*m  ->  d*sc*sum(q x) - dmin*m*sum(x)
// (src/kernels.c:414-510; get_scale_min_k4 include/quant.h:21-29)
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
__device__ __forceinline__ void blk_qk(const uint8_t* __restrict__ unit, const uint2* __restrict__ xf,
                                       const float* __restrict__ xsum_blk, int xsum_stride, int lane,
                                       float (&ab)[NT][4], float (&mt)[NT][4]) {
    const int g = lane >> 2, c = lane & 3;
    constexpr int QS = 2048, QH = 2048, SC = Q5 ? 2560 : 2048;
    const uint8_t* hdr_g = unit + SC + g * 16;
    const uint8_t* hdr_g8 = unit + SC + (g + 8) * 16;
    const uint4 hg = ldg_nc_128(hdr_g);
    const uint4 hg8 = ldg_nc_128(hdr_g8);
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
    if (Q5) qh = ldg_nc_128(unit + QH + lane * 16);   // [row g s0][row g s1][row g8 s0][row g8 s1]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        // words [row g s0][row g s1][row g8 s0][row g8 s1] of bytes 32j + 16s + 4c..
        const uint4 q = ldg_nc_128(unit + QS * 0 + j * 512 + lane * 16);
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
            const int sb = 2 * j + hi;
            float cs[NT][4];
#pragma unroll
            for (int ct = 0; ct < NT; ++ct) cs[ct][0] = cs[ct][1] = cs[ct][2] = cs[ct][3] = 0.f;
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
                mma_step<NT>(cs, a, xf + (sb * 2 + s) * NT * 32, lane);
            }
            float scg, mg, scg8, mg8;
            k4_scale_min(s12g, sb, scg, mg);
            k4_scale_min(s12g8, sb, scg8, mg8);
            scale_acc<NT>(ab, cs, dg * scg, dg8 * scg8);
            // - dmin*m * sum(x): x sums are unscaled, so this term goes to mt, which
            // is added to the result without the block's activation scale.
#pragma unroll
            for (int ct = 0; ct < NT; ++ct) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int col = 2 * c + i;
                    const bool is_lo = NT == 1 ? (col >= 4) : (ct == 1);
                    if (!is_lo) {
                        const int tok = col_token<NT>(ct, col);
                        const float xs = xsum_blk[tok * xsum_stride + sb];
                        mt[ct][i] -= dmg * mg * xs;
                        mt[ct][2 + i] -= dmg8 * mg8 * xs;
                    }
                }
            }
        }
    }
}

template <int NT>
__device__ __forceinline__ void blk_q6k(const uint8_t* __restrict__ unit, const uint2* __restrict__ xf,
                                        int lane, float (&ab)[NT][4]) {
    const int g = lane >> 2;
    // lo plane 2048 B: 4 chunks x 32 lanes x 16 B (one word per 16-element group)
    // hi plane 1024 B: 2 chunks x 32 lanes x 16 B (one word per pair of groups)
    // scales 256 B: [row][16] int8 ; d 32 B: [row] fp16
    const uint4 sc_g = ldg_nc_128(unit + 3072 + g * 16);
    const uint4 sc_g8 = ldg_nc_128(unit + 3072 + (g + 8) * 16);
    const uint32_t dd = __ldg(reinterpret_cast<const unsigned short*>(unit + 3328) + g) |
                        ((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(unit + 3328) + g + 8) << 16);
    const float dg = h2f_bits(dd), dg8 = h2f_bits(dd >> 16);
    const uint32_t scw_g[4] = {sc_g.x, sc_g.y, sc_g.z, sc_g.w};
    const uint32_t scw_g8[4] = {sc_g8.x, sc_g8.y, sc_g8.z, sc_g8.w};
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
        const uint4 hq = ldg_nc_128(unit + 2048 + ch * 512 + lane * 16);
        const uint32_t hw[4] = {hq.x, hq.y, hq.z, hq.w};
#pragma unroll
        for (int qc = 0; qc < 2; ++qc) {
            const uint4 lq = ldg_nc_128(unit + (ch * 2 + qc) * 512 + lane * 16);
            const uint32_t lw[4] = {lq.x, lq.y, lq.z, lq.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int G = (ch * 2 + qc) * 4 + i;       // 16-element group
                const uint32_t h = hw[G >> 1 & 3];           // word of groups (2m, 2m+1)
                const bool B = G & 1;
                const uint32_t he = B ? ((h << 4) & 0x30303030u) : (h & 0x30303030u);
                const uint32_t ho = B ? ((h << 2) & 0x30303030u) : ((h >> 2) & 0x30303030u);
                const uint32_t ev = (lw[i] & 0x0F0F0F0Fu) | he;          // [e0(g) e2(g) e0(g8) e2(g8)]
                const uint32_t od = ((lw[i] >> 4) & 0x0F0F0F0Fu) | ho;   // [e1(g) e3(g) e1(g8) e3(g8)]
                const uint32_t p01 = prmt(ev, od, 0x5140u);  // [e0g o0g e1g o1g] -> rows g: (e0,o0),(e1,o1)
                const uint32_t p23 = prmt(ev, od, 0x7362u);  // row g8
                uint32_t a[4];
                a[0] = hsub2_u32(prmt(p01, C64, 0x5140u), H1056x2);  // row g  elems 4c,4c+1
                a[2] = hsub2_u32(prmt(p01, C64, 0x7362u), H1056x2);  // row g  elems 4c+2,4c+3
                a[1] = hsub2_u32(prmt(p23, C64, 0x5140u), H1056x2);  // row g8
                a[3] = hsub2_u32(prmt(p23, C64, 0x7362u), H1056x2);
                float cs[NT][4];
#pragma unroll
                for (int ct = 0; ct < NT; ++ct) cs[ct][0] = cs[ct][1] = cs[ct][2] = cs[ct][3] = 0.f;
                // group G = sub-block G/2, step G&1
                mma_step<NT>(cs, a, xf + G * NT * 32, lane);
                const int scg = (int)(int8_t)(scw_g[G >> 2] >> (8 * (G & 3)));
                const int scg8 = (int)(int8_t)(scw_g8[G >> 2] >> (8 * (G & 3)));
                const float fg = dg * (small_u2f((uint32_t)(scg + 128)) - 128.f);
                const float fg8 = dg8 * (small_u2f((uint32_t)(scg8 + 128)) - 128.f);
                scale_acc<NT>(ab, cs, fg, fg8);
            }
        }
    }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(256) qmv_kernel(QmvParams p) {
    const int tile = blockIdx.x;
    int si = 0;
#pragma unroll
    for (int s = 1; s < QB_MAX_SEG; ++s)
        if (s < p.nseg && tile >= p.seg[s].tile0) si = s;
    const QSeg S = p.seg[si];
    const int lt = tile - S.tile0;
    const int nb = p.K >> 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int b0 = nb * warp / nw, b1 = nb * (warp + 1) / nw;
    constexpr int UB = FMT == QB_Q8_0 ? 8 * qb_unit_bytes(QB_Q8_0) : qb_unit_bytes(FMT);
    const uint8_t* base = S.w + (size_t)lt * nb * UB;

    float acc[NT][4];
#pragma unroll
    for (int ct = 0; ct < NT; ++ct) acc[ct][0] = acc[ct][1] = acc[ct][2] = acc[ct][3] = 0.f;

    for (int b = b0; b < b1; ++b) {
        float ab[NT][4], mt[NT][4];
#pragma unroll
        for (int ct = 0; ct < NT; ++ct) {
            ab[ct][0] = ab[ct][1] = ab[ct][2] = ab[ct][3] = 0.f;
            mt[ct][0] = mt[ct][1] = mt[ct][2] = mt[ct][3] = 0.f;
        }
        const uint8_t* unit = base + (size_t)b * UB;
        const uint2* xf = p.xfrag + (size_t)b * 16 * NT * 32;   // 8 sub-blocks x 2 steps
        if (FMT == QB_IQ4_XS) blk_iq4xs<NT>(unit, xf, lane, ab);
        else if (FMT == QB_Q8_0) blk_q8_0<NT>(unit, xf, lane, ab);
        else if (FMT == QB_Q4_K) blk_qk<NT, false>(unit, xf, p.xsum + b * 8, p.K >> 5, lane, ab, mt);
        else if (FMT == QB_Q5_K) blk_qk<NT, true>(unit, xf, p.xsum + b * 8, p.K >> 5, lane, ab, mt);
        else if (FMT == QB_Q6_K) blk_q6k<NT>(unit, xf, lane, ab);
#pragma unroll
        for (int ct = 0; ct < NT; ++ct) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int tok = col_token<NT>(ct, 2 * c + i);
                const float xs = __ldg(p.xscale + tok * nb + b);
                acc[ct][i] = fmaf(xs, ab[ct][i], acc[ct][i]) + mt[ct][i];
                acc[ct][2 + i] = fmaf(xs, ab[ct][2 + i], acc[ct][2 + i]) + mt[ct][2 + i];
            }
        }
    }

    // deterministic cross-warp reduction (warp order 0..nw-1)
    __shared__ float red[8][NT][4][32];
#pragma unroll
    for (int ct = 0; ct < NT; ++ct)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[warp][ct][i][lane] = acc[ct][i];
    __syncthreads();
    if (warp != 0) return;
    float v[NT][4];
#pragma unroll
    for (int ct = 0; ct < NT; ++ct)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float s = 0.f;
            for (int w = 0; w < nw; ++w) s += red[w][ct][i][lane];
            v[ct][i] = s;
        }
    // combine hi + lo columns
    float o[4];   // rows g (i=0,1) and g+8 (i=2,3); tokens t0 = tok(2c), t1 = tok(2c+1)
    int t0, t1;
    bool active;
    if (NT == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = v[0][i] + __shfl_xor_sync(0xffffffffu, v[0][i], 2);
        active = c < 2;
        t0 = 2 * c;
        t1 = 2 * c + 1;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = v[0][i] + v[NT - 1][i];
        active = true;
        t0 = 2 * c;
        t1 = 2 * c + 1;
    }
    if (!active) return;
    const int r0 = lt * QB_TILE + g, r1 = r0 + 8;
    const int rlo = p.row_lo, rhi = p.row_hi;
    auto store = [&](int t, int r, float val) {
        if (t < p.N && r < S.rows && r >= rlo && r < rhi) {
            float* dst = S.out + (size_t)t * S.ldo + r;
            *dst = p.accumulate ? (*dst + val) : val;
        }
    };
    store(t0, r0, o[0]);
    store(t1, r0, o[1]);
    store(t0, r1, o[2]);
    store(t1, r1, o[3]);
}

// ------------------------------- F32 ---------------------------------------
// Plain fp32 rows (src/kernels.c:342-357).  One warp per row.
__global__ void qmv_f32_kernel(const float* __restrict__ W, int rows, int K, const float* __restrict__ x,
                               long long ldx, int N, float* __restrict__ out, long long ldo, int accumulate,
                               int row_lo, int row_hi) {
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
// One warp per (tile, unit).  src rows are GGUF rows of row_bytes bytes.

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
    const int src_block = type == QB_Q8_0 ? 34 : UB / 16;
    auto rowp = [&](int rr) -> const uint8_t* {
        const int r = tile * QB_TILE + rr;
        return r < rows ? src + (size_t)r * row_bytes + (size_t)u * src_block : nullptr;
    };
    auto w32 = [&](const uint8_t* rp, int off) -> uint32_t { return rp ? ld_u32_unaligned(rp + off) : 0u; };
    const uint8_t* pg = rowp(g);
    const uint8_t* pg8 = rowp(g + 8);
    uint32_t* d32 = reinterpret_cast<uint32_t*>(d);

    if (type == QB_IQ4_XS) {
        // qs at byte 8 of the 136-byte block; sub-block sb = bytes 8+16sb..
        for (int p = 0; p < 4; ++p) {
            d32[(p * 512 + lane * 16) / 4 + 0] = w32(pg, 8 + 16 * (2 * p) + 4 * c);
            d32[(p * 512 + lane * 16) / 4 + 1] = w32(pg8, 8 + 16 * (2 * p) + 4 * c);
            d32[(p * 512 + lane * 16) / 4 + 2] = w32(pg, 8 + 16 * (2 * p + 1) + 4 * c);
            d32[(p * 512 + lane * 16) / 4 + 3] = w32(pg8, 8 + 16 * (2 * p + 1) + 4 * c);
        }
        if (lane < 16) {
            const uint8_t* rp = rowp(lane);
            d32[(2048 + lane * 8) / 4 + 0] = w32(rp, 0);
            d32[(2048 + lane * 8) / 4 + 1] = w32(rp, 4);
        }
    } else if (type == QB_Q8_0) {
        // block: d (2) + qs[32]; step s: elements 16s + 4c .. 16s + 4c + 3
        d32[lane * 4 + 0] = w32(pg, 2 + 4 * c);
        d32[lane * 4 + 1] = w32(pg8, 2 + 4 * c);
        d32[lane * 4 + 2] = w32(pg, 2 + 16 + 4 * c);
        d32[lane * 4 + 3] = w32(pg8, 2 + 16 + 4 * c);
        if (lane < 16) {
            const uint8_t* rp = rowp(lane);
            reinterpret_cast<uint16_t*>(d + 512)[lane] = rp ? (uint16_t)(rp[0] | (rp[1] << 8)) : 0;
        }
    } else if (type == QB_Q4_K || type == QB_Q5_K) {
        // block: d(2) dmin(2) scales(12) [qh(32) for Q5_K] qs(128)
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
        // block: ql[128] qh[64] scales[16] d(2).  Element e of group G (16G + l'):
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
        // lo plane: chunk qc (groups 4qc..4qc+3), word i = group G = 4qc+i:
        //   nibbles 0..3 = row g elements 4c..4c+3, nibbles 4..7 = row g8
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
        // hi plane: word for group pair (2m', 2m'+1), stored at chunk m'/4, slot m'%4.
        // byte j: bits 4-5 = A even_j, 6-7 = A odd_j, 0-1 = B even_j, 2-3 = B odd_j, where
        // even = (row g e0, row g e2, row g8 e0, row g8 e2), odd = (e1, e3 likewise).
        for (int mp = 0; mp < 8; ++mp) {
            uint32_t wv = 0;
            for (int j = 0; j < 4; ++j) {
                const uint8_t* rp = j < 2 ? pg : pg8;
                const int ee = (j & 1) ? 2 : 0;      // element offset of the even member
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
            for (int i = 0; i < 4; ++i) d32[(3072 + lane * 16) / 4 + i] = w32(rp, 192 + 4 * i);
            reinterpret_cast<uint16_t*>(d + 3328)[lane] = rp ? (uint16_t)(rp[208] | (rp[209] << 8)) : 0;
        }
    }
}

// ------------------------- activation fragments ------------------------------
// x [N][ldx] fp32 -> xfrag (hi/lo fp16, B-fragment order), xscale, xsum.
// Optional RMSNorm folded in: y = (x * inv_rms) * w  (src/kernels.c:741-777),
// with inv_rms computed per token by the same CTA.  Two segments allow the
// MTP concat [RMSNorm(e, enorm) || RMSNorm(h, hnorm)] (src/model.c:1044-1047).
// One CTA per (token, slice of 256-column blocks).

struct XSeg {
    const float* x;       // segment input, token t at x + t*ldx
    long long ldx;
    const float* w;       // RMSNorm weight (nullptr: no norm)
    int len;              // columns in this segment (multiple of 256)
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

__global__ void __launch_bounds__(256) xprep_kernel(XSeg s0, XSeg s1, int nseg, int N, int NT, float eps,
                                                    uint2* __restrict__ xfrag, float* __restrict__ xscale,
                                                    float* __restrict__ xsum, int want_xsum) {
    const int t = blockIdx.y;
    const int K = s0.len + (nseg > 1 ? s1.len : 0);
    const int nb = K >> 8;
    __shared__ float sh[32];
    float inv[2] = {1.f, 1.f};
    for (int si = 0; si < nseg; ++si) {
        const XSeg& S = si ? s1 : s0;
        if (!S.w) continue;
        const float* x = S.x + (size_t)t * S.ldx;
        float ss = 0.f;
        for (int i = threadIdx.x; i < S.len; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
        ss = block_sum(ss, sh);
        inv[si] = 1.0f / sqrtf(ss / (float)S.len + eps);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int ct_hi = 0;
    for (int b = blockIdx.x * nw + warp; b < nb; b += gridDim.x * nw) {
        const int col0 = b * 256;
        const int si = (nseg > 1 && col0 >= s0.len) ? 1 : 0;
        const XSeg& S = si ? s1 : s0;
        const int lc0 = col0 - (si ? s0.len : 0);
        const float* x = S.x + (size_t)t * S.ldx + lc0;
        float v[8];
        // lane owns elements 4*lane .. 4*lane+3 and 128 + 4*lane .. +3
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float4 xv = *reinterpret_cast<const float4*>(x + h * 128 + 4 * lane);
            v[4 * h + 0] = xv.x; v[4 * h + 1] = xv.y; v[4 * h + 2] = xv.z; v[4 * h + 3] = xv.w;
            if (S.w) {
                const float4 wv = *reinterpret_cast<const float4*>(S.w + lc0 + h * 128 + 4 * lane);
                v[4 * h + 0] = (v[4 * h + 0] * inv[si]) * wv.x;
                v[4 * h + 1] = (v[4 * h + 1] * inv[si]) * wv.y;
                v[4 * h + 2] = (v[4 * h + 2] * inv[si]) * wv.z;
                v[4 * h + 3] = (v[4 * h + 3] * inv[si]) * wv.w;
            }
        }
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
        for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        int e = 0;
        if (am > 0.f && isfinite(am)) {
            int ex;
            frexpf(am, &ex);          // am in [2^(ex-1), 2^ex)
            e = 15 - ex;              // am * 2^e in [2^14, 2^15)
            e = max(-100, min(100, e));
        }
        if (lane == 0) xscale[t * nb + b] = ldexpf(1.f, -e);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            // elements col0 + h*128 + 4*lane + k  -> sub-block, step, quad thread
            const int el = h * 128 + 4 * lane;          // within the 256-block
            const int sb = b * 8 + (el >> 5), st = (el >> 4) & 1, cq = (el >> 2) & 3;
            __half hv[4], lv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float xs = ldexpf(v[4 * h + k], e);
                hv[k] = __float2half_rn(xs);
                lv[k] = __float2half_rn(xs - __half2float(hv[k]));
            }
            uint2 hi, lo;
            hi.x = (uint32_t)__half_as_ushort(hv[0]) | ((uint32_t)__half_as_ushort(hv[1]) << 16);
            hi.y = (uint32_t)__half_as_ushort(hv[2]) | ((uint32_t)__half_as_ushort(hv[3]) << 16);
            lo.x = (uint32_t)__half_as_ushort(lv[0]) | ((uint32_t)__half_as_ushort(lv[1]) << 16);
            lo.y = (uint32_t)__half_as_ushort(lv[2]) | ((uint32_t)__half_as_ushort(lv[3]) << 16);
            int col_hi, col_lo, cth, ctl;
            if (NT == 1) { col_hi = t; col_lo = t + 4; cth = ctl = 0; }
            else { col_hi = t; col_lo = t; cth = ct_hi; ctl = 1; }
            const size_t base = (size_t)(sb * 2 + st) * NT;
            xfrag[(base + cth) * 32 + col_hi * 4 + cq] = hi;
            xfrag[(base + ctl) * 32 + col_lo * 4 + cq] = lo;
            if (want_xsum) {
                // sum of the 32 unscaled elements of sub-block sb: 8 lanes hold it
                float ps = v[4 * h] + v[4 * h + 1] + v[4 * h + 2] + v[4 * h + 3];
                ps += __shfl_xor_sync(0xffffffffu, ps, 1);
                ps += __shfl_xor_sync(0xffffffffu, ps, 2);
                ps += __shfl_xor_sync(0xffffffffu, ps, 4);
                if ((lane & 7) == 0) xsum[t * (K >> 5) + sb] = ps;
            }
        }
    }
}

}  // namespace

// ============================ host launchers ==================================

static const uint8_t kIq4Lut[16] = {
    // kvalues_iq4nl + 128
    1, 24, 45, 63, 79, 93, 106, 118, 129, 141, 153, 166, 181, 197, 217, 241,
};

cudaError_t qb_quant_init_constants() {
    uint32_t w[4];
    for (int i = 0; i < 4; ++i)
        w[i] = kIq4Lut[4 * i] | (kIq4Lut[4 * i + 1] << 8) | (kIq4Lut[4 * i + 2] << 16) |
               ((uint32_t)kIq4Lut[4 * i + 3] << 24);
    return cudaMemcpyToSymbol(c_iq4_lut, w, sizeof w);
}

size_t qb_repacked_bytes(int type, int rows, int K) {
    const int ub = qb_unit_bytes(type), uc = qb_unit_cols(type);
    if (!ub || K % 256) return 0;
    const size_t tiles = (size_t)(rows + QB_TILE - 1) / QB_TILE;
    return tiles * (size_t)(K / uc) * ub;
}

cudaError_t qb_repack(int type, const void* src_dev, int rows, int K, void* dst_dev, cudaStream_t st) {
    const int ub = qb_unit_bytes(type), uc = qb_unit_cols(type);
    if (!ub || K % 256) return cudaErrorInvalidValue;
    const int upr = K / uc;
    const size_t row_bytes = (size_t)upr * (type == QB_Q8_0 ? 34 : ub / 16);
    const long long tiles = (rows + QB_TILE - 1) / QB_TILE;
    const long long units = tiles * upr;
    const int threads = 256;
    const long long blocks = (units * 32 + threads - 1) / threads;
    repack_kernel<<<(unsigned)blocks, threads, 0, st>>>(type, (const uint8_t*)src_dev, row_bytes, rows, upr,
                                                        (uint8_t*)dst_dev, units);
    return cudaGetLastError();
}

cudaError_t qb_xprep(const QbXIn* in, int nseg, int N, float eps, uint2* xfrag, float* xscale, float* xsum,
                     int want_xsum, cudaStream_t st) {
    XSeg s[2] = {};
    int K = 0;
    for (int i = 0; i < nseg; ++i) {
        s[i].x = in[i].x;
        s[i].ldx = in[i].ldx;
        s[i].w = in[i].norm_w;
        s[i].len = in[i].len;
        if (in[i].len % 256) return cudaErrorInvalidValue;
        K += in[i].len;
    }
    const int NT = N <= 4 ? 1 : 2;
    const int nb = K / 256;
    const int any_norm = (s[0].w != nullptr) || (nseg > 1 && s[1].w != nullptr);
    // with a norm the per-token reduction needs the whole token in one CTA
    const int gx = any_norm ? 1 : (nb + 7) / 8;
    xprep_kernel<<<dim3(gx, N), 256, 0, st>>>(s[0], s[1], nseg, N, NT, eps, xfrag, xscale, xsum, want_xsum);
    return cudaGetLastError();
}

cudaError_t qb_qmv(int type, const QbQSeg* segs, int nseg, int K, int N, const uint2* xfrag,
                   const float* xscale, const float* xsum, int accumulate, int row_lo, int row_hi,
                   cudaStream_t st) {
    if (nseg < 1 || nseg > QB_MAX_SEG || N < 1 || N > QB_MAX_TOK || K % 256) return cudaErrorInvalidValue;
    QmvParams p = {};
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        p.seg[i].w = (const uint8_t*)segs[i].w;
        p.seg[i].out = segs[i].out;
        p.seg[i].ldo = segs[i].ldo;
        p.seg[i].rows = segs[i].rows;
        p.seg[i].tile0 = tiles;
        tiles += (segs[i].rows + QB_TILE - 1) / QB_TILE;
    }
    p.nseg = nseg;
    p.K = K;
    p.N = N;
    p.xfrag = xfrag;
    p.xscale = xscale;
    p.xsum = xsum;
    p.accumulate = accumulate;
    p.row_lo = row_lo;
    p.row_hi = row_hi;
    // K split across warps of the CTA: more warps when there are few tiles
    const int nb = K / 256;
    int warps = tiles >= 1024 ? 4 : 8;
    if (warps > nb) warps = nb;
    const dim3 grid(tiles), block(32 * warps);
    const bool nt2 = N > 4;
#define QB_LAUNCH(F)                                                             \
    do {                                                                         \
        if (nt2) qmv_kernel<F, 2><<<grid, block, 0, st>>>(p);                    \
        else qmv_kernel<F, 1><<<grid, block, 0, st>>>(p);                        \
    } while (0)
    switch (type) {
    case QB_IQ4_XS: QB_LAUNCH(QB_IQ4_XS); break;
    case QB_Q8_0: QB_LAUNCH(QB_Q8_0); break;
    case QB_Q4_K: QB_LAUNCH(QB_Q4_K); break;
    case QB_Q5_K: QB_LAUNCH(QB_Q5_K); break;
    case QB_Q6_K: QB_LAUNCH(QB_Q6_K); break;
    default: return cudaErrorInvalidValue;
    }
#undef QB_LAUNCH
    return cudaGetLastError();
}

cudaError_t qb_qmv_f32(const float* W, int rows, int K, const float* x, long long ldx, int N, float* out,
                       long long ldo, int accumulate, int row_lo, int row_hi, cudaStream_t st) {
    const int n = row_hi - row_lo;
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    const int blocks = (n * 32 + threads - 1) / threads;
    qmv_f32_kernel<<<blocks, threads, 0, st>>>(W, rows, K, x, ldx, N, out, ldo, accumulate, row_lo, row_hi);
    return cudaGetLastError();
}
