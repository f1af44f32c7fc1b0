// Activation preparation for the quantised GEMV, shared by xprep_kernel and
// the kernels that produce a GEMV input (SwiGLU, gated RMSNorm, attention):
// one warp turns one 256-column block of one token into the B fragments the
// GEMV reads (qb_kernels.h QbXBuf).
#pragma once
#include "qb_common.cuh"
#include "qb_kernels.h"

// v[0..3] = elements 4*lane .. 4*lane+3 of the block, v[4..7] = 128 + 4*lane ..;
// t = token, b = block index, N tokens in the launch, nb = K / 256 blocks.
__device__ __forceinline__ void xprep_emit(const float (&v)[8], int t, int b, int N, int nb, int K,
                                           const QbXBuf& xb, int what, int lane) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    int ex = 0;
    const bool nz = am > 0.f && isfinite(am);
    if (nz) frexpf(am, &ex);   // am < 2^ex
    if (what & QB_XP_F16) {
        const int NT = N <= 4 ? 1 : 2;
        const int e = nz ? max(-100, min(100, 15 - ex)) : 0;   // am * 2^e in [2^14, 2^15)
        if (lane == 0) xb.xscale[t * nb + b] = ldexpf(1.f, -e);
        const float sc = ldexpf(1.f, e);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int el = h * 128 + 4 * lane;
            const int sb = b * 8 + (el >> 5), st = (el >> 4) & 1, cq = (el >> 2) & 3;
            __half hv[4], lv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float xs = v[4 * h + k] * sc;
                hv[k] = __float2half_rn(xs);
                lv[k] = __float2half_rn(xs - __half2float(hv[k]));
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
    if (what & QB_XP_SUM) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int sb = b * 8 + ((h * 128 + 4 * lane) >> 5);
            float ps = v[4 * h] + v[4 * h + 1] + v[4 * h + 2] + v[4 * h + 3];
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            if ((lane & 7) == 0) xb.xsum[t * (K >> 5) + sb] = ps;
        }
    }
    if (what & (QB_XP_I8 | QB_XP_TC)) {
        // X = rint(x * 2^e) with |X| <= 2^22, as balanced int8 digits X = 65536 d0 + 256 d1 + d2
        // (|d0| <= 64).  Lane 8j + c (c < 4) holds elements 4c..4c+3 of sub-block j and
        // lane 8j + c + 4 elements 16+4c..16+4c+3: together one mma B register pair.
        const int NTI = N <= 4 ? 2 : 3;
        const int e = nz ? max(-120, min(120, 22 - ex)) : 0;
        if (lane == 0) xb.xqscale[t * nb + b] = ldexpf(1.f, -e);
        const float sc = ldexpf(1.f, e);
        const int c = lane & 3;
        const bool first = (lane & 4) == 0;
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
        for (int h = 0; h < 2; ++h) {
            uint32_t dg[3] = {0u, 0u, 0u};   // per digit: 4 bytes, element order 0..3 of this lane
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int X = __float2int_rn(v[4 * h + k] * sc);
                const int d2 = (int)(int8_t)(X & 0xFF);
                const int X1 = (X - d2) >> 8;
                const int d1 = (int)(int8_t)(X1 & 0xFF);
                const int d0 = (X1 - d1) >> 8;
                dg[0] |= ((uint32_t)d0 & 0xFFu) << (8 * k);
                dg[1] |= ((uint32_t)d1 & 0xFFu) << (8 * k);
                dg[2] |= ((uint32_t)d2 & 0xFFu) << (8 * k);
            }
            const int kb = b * 8 + h * 4 + (lane >> 3);   // global sub-block (k32) index
#pragma unroll
            for (int dgi = 0; dgi < 3; ++dgi) {
                const uint32_t other = __shfl_xor_sync(0xffffffffu, dg[dgi], 4);
                if (first) {
                    uint2 bv;
                    bv.x = prmt(dg[dgi], other, 0x5140u);   // (4c, 4c+16, 4c+1, 4c+17)
                    bv.y = prmt(dg[dgi], other, 0x7362u);   // (4c+2, 4c+18, 4c+3, 4c+19)
                    if (what & QB_XP_I8) xb.xq[((size_t)kb * NTI + dnt[dgi]) * 32 + dcol[dgi] * 4 + c] = bv;
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
