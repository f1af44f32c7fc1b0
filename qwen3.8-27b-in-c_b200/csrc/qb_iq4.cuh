// IQ4_XS decode helpers of the mma.sync GEMV (iq4_pq) and of the tcgen05 variant
// (iq4_scale_bytes, iq4_i8).
//
// Scales in the tcgen05 tile (the mma.sync tile stores the sub-block scales as
// int8 differences instead, qb_quant.cu): each row of a 256-column block keeps its 8 bytes of scales as
// [A(4) d(2) Bh(2)]: A byte i = ls_i | (ls_{4+i} & 3) << 6, Bh nibble j =
// ls_{4+j} >> 2, d = the fp16 super-block scale (a byte-aligned rearrangement
// of block_iq4_xs scales_l / scales_h, include/quant.h:56-62; the 6-bit
// sub-scale ls_ib = scales_l nibble ib | scales_h bits 2ib..2ib+1 << 4,
// src/kernels.c:84-90).
//
// Codes: a 32-bit word holds qs bytes 4c..4c+3 of one row's sub-block, i.e.
// elements 4c..4c+3 (low nibbles) and 16+4c..16+4c+3 (high nibbles)
// (src/quant.c:175-176).
#pragma once
#include "qb_common.cuh"

// L0 = bytes ls_0..ls_3, L1 = bytes ls_4..ls_7, d = fp16 scale as float
__device__ __forceinline__ void iq4_scale_bytes(uint2 v, uint32_t& L0, uint32_t& L1, float& d) {
    L0 = v.x & 0x3F3F3F3Fu;
    const uint32_t x = prmt(v.y, 0u, 0x3322u);
    const uint32_t nib = (x & 0x000F000Fu) | ((x >> 4) & 0x0F000F00u);
    L1 = ((v.x >> 6) & 0x03030303u) | (nib << 2);
    d = h2f_bits(v.y);
}

// kvalues_iq4nl (src/quant.c:30-32) as int8, four per word
constexpr uint32_t kIq4I8T0 = 0xBFAD9881u;   // -127 -104  -83  -65
constexpr uint32_t kIq4I8T1 = 0xF6EADDCFu;   //  -49  -35  -22  -10
constexpr uint32_t kIq4I8T2 = 0x26190D01u;   //    1   13   25   38
constexpr uint32_t kIq4I8T3 = 0x71594535u;   //   53   69   89  113

// 8 codes -> int8 values: lo = elements (4c, 4c+16, 4c+1, 4c+17),
// hi = (4c+2, 4c+18, 4c+3, 4c+19).  Two 8-entry byte-permute lookups per 4
// codes and a select on code bit 3.
__device__ __forceinline__ void iq4_i8(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t idx = w & 0x77777777u;                         // table index, code bit 3 cleared
    const uint32_t sel = ((w >> 1) & 0x44444444u) | 0x32103210u;  // code bit 3 picks the upper table
    const uint32_t idxh = idx >> 16, selh = sel >> 16;
    lo = prmt(prmt(kIq4I8T0, kIq4I8T1, idx), prmt(kIq4I8T2, kIq4I8T3, idx), sel);
    hi = prmt(prmt(kIq4I8T0, kIq4I8T1, idxh), prmt(kIq4I8T2, kIq4I8T3, idxh), selh);
}

// The same 8 codes as two int8 terms P + Q = the table value, with no select:
// a byte-permute selector nibble with bit 3 set yields the selected byte's sign
// replicated.  P looks up values 0..7 (all negative) with the code itself as
// the selector: codes 8..15 give -1.  Q looks up values 8..15 plus 1 (all
// positive) with code ^ 8: codes 0..7 give 0.  Two mma steps then sum P and Q.
constexpr uint32_t kIq4QT2 = 0x271A0E02u;   //  2 14 26  39  (values 8..11, plus 1)
constexpr uint32_t kIq4QT3 = 0x725A4636u;   // 54 70 90 114  (values 12..15, plus 1)
__device__ __forceinline__ void iq4_pq(uint32_t w, uint32_t& plo, uint32_t& phi, uint32_t& qlo, uint32_t& qhi) {
    const uint32_t x = w ^ 0x88888888u;
    plo = prmt(kIq4I8T0, kIq4I8T1, w);
    phi = prmt(kIq4I8T0, kIq4I8T1, w >> 16);
    qlo = prmt(kIq4QT2, kIq4QT3, x);
    qhi = prmt(kIq4QT2, kIq4QT3, x >> 16);
}

// byte i of w, sign-extended
__device__ __forceinline__ int sbyte(uint32_t w, int i) {
    return (int)prmt(w, 0u, (uint32_t)(i | ((8 | i) << 4) | ((8 | i) << 8) | ((8 | i) << 12)));
}

// byte i of w, zero-extended
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)prmt(w, 0u, (uint32_t)(0x4440 | i)); }
