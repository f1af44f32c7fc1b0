// Activation preparation for the quantised GEMV, shared by xprep_kernel and
// the kernels that produce a GEMV input (SwiGLU, gated RMSNorm, attention):
// one warp turns one 256-column block of one token into the B fragments the
// GEMV reads (qb_kernels.h QbXBuf).
#pragma once
#include "qb_common.cuh"
#include "qb_kernels.h"

// v[k][0..3] = elements 4*lane .. 4*lane+3 of the block for token t0 + k,
// v[k][4..7] = 128 + 4*lane ..; b = block index, N tokens in the launch,
// nb = K / 256 blocks.  The G tokens go through every step together, so
// their shuffle / convert chains interleave.
template <int G>
__device__ __forceinline__ void xprep_emit_g(const float (&v)[G][8], int t0, int b, int N, int nb, int K,
                                             const QbXBuf& xb, int what, int lane) {
    int ex[G];
    bool nz[G];
    {
        float am[G];
#pragma unroll
        for (int k = 0; k < G; ++k) {
            am[k] = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) am[k] = fmaxf(am[k], fabsf(v[k][i]));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1)
#pragma unroll
            for (int k = 0; k < G; ++k) am[k] = fmaxf(am[k], __shfl_xor_sync(0xffffffffu, am[k], o));
#pragma unroll
        for (int k = 0; k < G; ++k) {
            ex[k] = 0;
            nz[k] = am[k] > 0.f && isfinite(am[k]);
            if (nz[k]) frexpf(am[k], &ex[k]);   // am < 2^ex
        }
    }
    if (what & QB_XP_F16) {
        const int NT = N <= 4 ? 1 : 2;
#pragma unroll
        for (int k = 0; k < G; ++k) {
            const int t = t0 + k;
            const int e = nz[k] ? max(-100, min(100, 15 - ex[k])) : 0;   // am * 2^e in [2^14, 2^15)
            if (lane == 0) xb.xscale[t * nb + b] = ldexpf(1.f, -e);
            const float sc = ldexpf(1.f, e);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int el = h * 128 + 4 * lane;
                const int sb = b * 8 + (el >> 5), st = (el >> 4) & 1, cq = (el >> 2) & 3;
                __half hv[4], lv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float xs = v[k][4 * h + j] * sc;
                    hv[j] = __float2half_rn(xs);
                    lv[j] = __float2half_rn(xs - __half2float(hv[j]));
                }
                uint2 hi, lo;
                hi.x = (uint32_t)__half_as_ushort(hv[0]) | ((uint32_t)__half_as_ushort(hv[1]) << 16);
                hi.y = (uint32_t)__half_as_ushort(hv[2]) | ((uint32_t)__half_as_ushort(hv[3]) << 16);
                lo.x = (uint32_t)__half_as_ushort(lv[0]) | ((uint32_t)__half_as_ushort(lv[1]) << 16);
                lo.y = (uint32_t)__half_as_ushort(lv[2]) | ((uint32_t)__half_as_ushort(lv[3]) << 16);
                const size_t base = (size_t)(sb * 2 + st) * NT;
                if (NT == 1) {
                    xb.xfrag[base * 32 + t * 4 + cq] = hi;
                    xb.xfrag[base * 32 + (t + 4) * 4 + cq] = lo;
                } else {
                    xb.xfrag[base * 32 + t * 4 + cq] = hi;
                    xb.xfrag[(base + 1) * 32 + t * 4 + cq] = lo;
                }
            }
        }
    }
    if (what & QB_XP_SUM) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int sb = b * 8 + ((h * 128 + 4 * lane) >> 5);
            float ps[G];
#pragma unroll
            for (int k = 0; k < G; ++k) ps[k] = v[k][4 * h] + v[k][4 * h + 1] + v[k][4 * h + 2] + v[k][4 * h + 3];
#pragma unroll
            for (int o = 1; o <= 4; o <<= 1)
#pragma unroll
                for (int k = 0; k < G; ++k) ps[k] += __shfl_xor_sync(0xffffffffu, ps[k], o);
            if ((lane & 7) == 0)
#pragma unroll
                for (int k = 0; k < G; ++k) xb.xsum[(t0 + k) * (K >> 5) + sb] = ps[k];
        }
    }
    if (what & (QB_XP_I8 | QB_XP_TC | QB_XP_TC16 | QB_XP_TC32)) {
        // X = rint(x * 2^e) with |X| <= 2^22, as balanced int8 digits X = 65536 d0 + 256 d1 + d2
        // (|d0| <= 64).  Lane 8j + c (c < 4) holds elements 4c..4c+3 of sub-block j and
        // lane 8j + c + 4 elements 16+4c..16+4c+3: together one mma B register pair.
        const int NTI = N <= 4 ? 2 : 3;
        const int c = lane & 3;
        const bool first = (lane & 4) == 0;
        float sc[G];
#pragma unroll
        for (int k = 0; k < G; ++k) {
            const int e = nz[k] ? max(-120, min(120, 22 - ex[k])) : 0;
            if (lane == 0) xb.xqscale[(t0 + k) * nb + b] = ldexpf(1.f, -e);
            sc[k] = ldexpf(1.f, e);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kb = b * 8 + h * 4 + (lane >> 3);   // global sub-block (k32) index
            uint32_t dg[G][3];   // per token and digit: 4 bytes, element order 0..3 of this lane
#pragma unroll
            for (int k = 0; k < G; ++k) {
                dg[k][0] = dg[k][1] = dg[k][2] = 0u;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int X = __float2int_rn(v[k][4 * h + j] * sc[k]);
                    const int d2 = (int)(int8_t)(X & 0xFF);
                    const int X1 = (X - d2) >> 8;
                    const int d1 = (int)(int8_t)(X1 & 0xFF);
                    const int d0 = (X1 - d1) >> 8;
                    dg[k][0] |= ((uint32_t)d0 & 0xFFu) << (8 * j);
                    dg[k][1] |= ((uint32_t)d1 & 0xFFu) << (8 * j);
                    dg[k][2] |= ((uint32_t)d2 & 0xFFu) << (8 * j);
                }
            }
            uint32_t other[G][3];
#pragma unroll
            for (int k = 0; k < G; ++k)
#pragma unroll
                for (int dgi = 0; dgi < 3; ++dgi) other[k][dgi] = __shfl_xor_sync(0xffffffffu, dg[k][dgi], 4);
            if (first) {
#pragma unroll
                for (int k = 0; k < G; ++k) {
                    const int t = t0 + k;
                    // destination (n8 tile, column) of each digit of token t
                    int dnt[3], dcol[3];
                    if (t < 4) {
                        dnt[0] = 0; dcol[0] = 2 * t;
                        dnt[1] = 0; dcol[1] = 2 * t + 1;
                        dnt[2] = 1; dcol[2] = 2 * t;
                    } else {
                        dnt[0] = 2; dcol[0] = 2 * (t - 4);
                        dnt[1] = 2; dcol[1] = 2 * (t - 4) + 1;
                        dnt[2] = 1; dcol[2] = 2 * (t - 4) + 1;
                    }
#pragma unroll
                    for (int dgi = 0; dgi < 3; ++dgi) {
                        uint2 bv;
                        bv.x = prmt(dg[k][dgi], other[k][dgi], 0x5140u);   // (4c, 4c+16, 4c+1, 4c+17)
                        bv.y = prmt(dg[k][dgi], other[k][dgi], 0x7362u);   // (4c+2, 4c+18, 4c+3, 4c+19)
                        if ((what & QB_XP_I8) && t < QB_MAX_TOK)
                            xb.xq[((size_t)kb * NTI + dnt[dgi]) * 32 + dcol[dgi] * 4 + c] = bv;
                        if ((what & QB_XP_TC16) && t < 16) {
                            // 48-row tcgen05 B tile of the sub-block, digit-major: row n = 16 digit + t
                            // (one 16-column accumulator group per digit); same core-matrix layout
                            const int nrow = 16 * dgi + t;
                            *reinterpret_cast<uint2*>(xb.xtc16 + (size_t)kb * 1536 + (c >> 1) * 128 +
                                                      (nrow >> 3) * 256 + (nrow & 7) * 16 + (c & 1) * 8) = bv;
                        }
                        if (what & QB_XP_TC32) {   // the same with 32 tokens: row n = 32 digit + t
                            const int nrow = 32 * dgi + t;
                            *reinterpret_cast<uint2*>(xb.xtc32 + (size_t)kb * 3072 + (c >> 1) * 128 +
                                                      (nrow >> 3) * 256 + (nrow & 7) * 16 + (c & 1) * 8) = bv;
                        }
                        if ((what & QB_XP_TC) && t < 4) {
                            // tcgen05 B tile of the sub-block: row n = 3t + digit, 32 k bytes in the
                            // order above; K-major core matrices of 8 rows x 16 B, K chunks 128 B apart,
                            // 8-row groups 256 B apart
                            const int nrow = 3 * t + dgi;
                            *reinterpret_cast<uint2*>(xb.xtc + (size_t)kb * 512 + (c >> 1) * 128 + (nrow >> 3) * 256 +
                                                      (nrow & 7) * 16 + (c & 1) * 8) = bv;
                        }
                    }
                }
            }
        }
    }
}

// one token: v[0..3] = elements 4*lane .. 4*lane+3 of block b of token t, v[4..7] = 128 + 4*lane ..
// A wide input (N > QB_MAX_TOK): the 8-row formats go to the chunk of 8 rows that
// holds t, the 16- / 32-token tcgen05 tiles take row t itself.
__device__ __forceinline__ void xprep_emit(const float (&v)[8], int t, int b, int N, int nb, int K,
                                           const QbXBuf& xb, int what, int lane) {
    const float (&v1)[1][8] = reinterpret_cast<const float (&)[1][8]>(v);
    if (N > QB_MAX_TOK) {
        const int tcw = what & (QB_XP_TC16 | QB_XP_TC32);
        const int rest = what & (QB_XP_F16 | QB_XP_SUM | QB_XP_I8);
        if (rest) {
            const int c = t >> 3;
            xprep_emit_g<1>(v1, t & 7, b, min(QB_MAX_TOK, N - 8 * c), nb, K, qb_xb_chunk(xb, c, nb), rest, lane);
        }
        if (tcw) xprep_emit_g<1>(v1, t, b, N, nb, K, xb, tcw, lane);
        return;
    }
    xprep_emit_g<1>(v1, t, b, N, nb, K, xb, what, lane);
}
