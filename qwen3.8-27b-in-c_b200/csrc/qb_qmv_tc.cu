// IQ4_XS GEMV on the sm_100a tcgen05 tensor cores, for N <= 4 input vectors
// (the verify width k+1 = 4 and the single-token drafts).
//
// Reference: dot_iq4_xs_b / gemv_rows_batch, src/kernels.c:373-412, 570-599;
// block format include/quant.h:56-62, values src/quant.c:30-32, 175-176.
//
// Data path per (128-row tile, 256-column block) stage:
//   * a producer warp bulk-copies the stage's 17408 weight bytes and the
//     block's 4 KB of activation digits into a shared-memory ring;
//   * four decode warps, one thread per weight row, turn the row's 256 codes
//     into int8 values (byte-permute table lookup) and store them to tensor
//     memory: lane = row, 4 values per 32-bit column, 8 columns per 32-column
//     sub-block;
//   * one thread issues eight tcgen05.mma.kind::i8 (M 128, N 16, K 32), one
//     per sub-block, each into its own 16 accumulator columns: A from tensor
//     memory, B = the digits (token t, digit d at row 3t + d) from shared
//     memory, exact int32 sums;
//   * one stage later the decode threads read their row's accumulators back
//     (tcgen05.ld), apply the 6-bit sub-block scales in int32, combine the
//     digits (X = 65536 d0 + 256 d1 + d2) and the fp16 block scale in fp32.
// The decode of stage r overlaps the MMAs of stage r-1.  Stages of all fused
// matrices are split evenly over the CTAs (stream-K); a tile split across
// CTAs is finished per row by the last contributing CTA, which sums the
// partials in CTA order (deterministic).  Every wait is bounded; on a
// time-out the kernel records an error, drains its copies and MMAs, frees
// its tensor memory and returns.
#include "qb_common.cuh"
#include "qb_kernels.h"
#include "qb_iq4.cuh"
#include "qb_tc.cuh"

namespace {

constexpr int kRows = 128;                  // rows per tile = tensor-memory lanes
constexpr int kUnit = kRows * 136;          // repacked bytes of one (tile, block)
constexpr int kQsBytes = kRows * 128;       // [8 sub-blocks][128 rows][16 B]
constexpr int kBBytes = 4096;               // activation digits of one block
constexpr int kStage = kUnit + kBBytes;     // 21504
constexpr int kRing = 4;
constexpr int kDecodeWarps = 4;
constexpr int kDecodeThreads = kDecodeWarps * 32;
constexpr int kThreads = kDecodeThreads + 32;   // + producer warp
constexpr int kCtasPerSm = 2;               // 2 x 256 tensor-memory columns = all 512
constexpr uint32_t kCols = 256;             // A: 2 x 64 columns, D: 8 sub-blocks x 16 columns
constexpr uint32_t kDCol = 128;
constexpr int kHdr = 256;
constexpr uint32_t kIdesc = idesc_i8(128, 16);
#ifndef QB_TC_SLEEP_NS
#define QB_TC_SLEEP_NS 2000
#endif
constexpr uint32_t kSleepNs = QB_TC_SLEEP_NS;   // suspend hint of the mbarrier waits (bounded: 2^16 tries)

struct TcK {
    const uint8_t* w[QB_MAX_SEG];   // tile-repacked weights of each fused matrix
    float* out[QB_MAX_SEG];
    long long ldo[QB_MAX_SEG];
    int rows[QB_MAX_SEG];
    int tile0[QB_MAX_SEG + 1];      // first tile of each matrix; tile0[nseg] = tiles
    int nseg, nb, N, S, G;          // S = tiles * nb stages over G CTAs
    const uint8_t* xb;              // activation digits, kBBytes per block
    const float* xqscale;           // [QB_MAX_TOK][nb]
    int accumulate, row_lo, row_hi;
    float* partial;                 // [G][2][kRows][4]
    unsigned* counters;             // [tiles][kRows], zero between launches
    unsigned* err;
};

__device__ __forceinline__ int cta_s0(int S, int G, int c) { return (int)((long long)S * c / G); }
__device__ __forceinline__ int stage_cta(int S, int G, int s) { return (int)(((long long)(s + 1) * G - 1) / S); }

__device__ __forceinline__ int seg_of_tile(const TcK& p, int T) {
    int sg = 0;
#pragma unroll
    for (int i = 1; i < QB_MAX_SEG; ++i)
        if (i < p.nseg && T >= p.tile0[i]) sg = i;
    return sg;
}

// row m of tile T is complete in this CTA's tot[]: store it, or combine the
// split tile's per-CTA partials (last arriving CTA, CTA order)
__device__ void finish_row(const TcK& p, int T, int cta, int s0, int s1, int m, const float (&tot)[4]) {
    const int sg = seg_of_tile(p, T);
    const int row = (T - p.tile0[sg]) * kRows + m;
    auto store = [&](const float (&v)[4]) {
        if (row >= p.rows[sg] || row < p.row_lo || row >= p.row_hi) return;
#pragma unroll
        for (int t = 0; t < 4; ++t)
            if (t < p.N) {
                float* dst = p.out[sg] + (size_t)t * p.ldo[sg] + row;
                *dst = p.accumulate ? (*dst + v[t]) : v[t];
            }
    };
    const int P0 = T * p.nb, P1 = P0 + p.nb;
    if (s0 <= P0 && s1 >= P1) {
        store(tot);
        return;
    }
    const int piece = s0 > P0 ? 0 : 1;   // 0: the tile is this CTA's first (it started inside it)
    *reinterpret_cast<float4*>(p.partial + (((size_t)cta * 2 + piece) * kRows + m) * 4) =
        make_float4(tot[0], tot[1], tot[2], tot[3]);
    const int c_first = stage_cta(p.S, p.G, P0), c_last = stage_cta(p.S, p.G, P1 - 1);
    unsigned* ctr = p.counters + (size_t)T * kRows + m;
    // release orders this thread's partial before the count, acquire the others' after it
    const unsigned old = atom_add_acq_rel_gpu(ctr, 1u);
    if ((int)old != c_last - c_first) return;
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = c_first; c <= c_last; ++c) {
        const int pc = cta_s0(p.S, p.G, c) > P0 ? 0 : 1;
        const volatile float* v = p.partial + (((size_t)c * 2 + pc) * kRows + m) * 4;
#pragma unroll
        for (int t = 0; t < 4; ++t) sum[t] += v[t];
    }
    store(sum);
    *ctr = 0u;   // ready for the next launch
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm) qmv_tc_kernel(TcK p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kRing;
    uint64_t* mma_done = empty + kRing;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* dec_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
    uint8_t* ring = smem + kHdr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int s0 = cta_s0(p.S, p.G, cta), s1 = cta_s0(p.S, p.G, cta + 1);
    const int n = s1 - s0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRing; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_init(mma_done, 1);
        *dec_abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    pdl_trigger();

    if (warp == kDecodeWarps) {
        // ------------------------------ producer ------------------------------
        if (lane == 0 && n > 0) {
            auto weights_of = [&](int s) -> const uint8_t* {
                const int T = s / p.nb, b = s - T * p.nb;
                const int sg = seg_of_tile(p, T);
                return p.w[sg] + ((size_t)(T - p.tile0[sg]) * p.nb + b) * kUnit;
            };
            const int pre = n < kRing ? n : kRing;
            // weights do not depend on the previous kernel: start streaming them before the wait
            for (int r = 0; r < pre; ++r) {
                mbar_expect_tx(full + r, kStage);
                bulk_g2s(ring + r * kStage, weights_of(s0 + r), kUnit, full + r);
            }
            pdl_wait();   // the activation digits are written by the previous kernel
            for (int r = 0; r < pre; ++r)
                bulk_g2s(ring + r * kStage + kUnit, p.xb + (size_t)((s0 + r) % p.nb) * kBBytes, kBBytes, full + r);
            int issued = pre;
            for (int r = kRing; r < n; ++r) {
                const int slot = r % kRing;
                if (!mbar_wait_sleep(empty + slot, (uint32_t)((r / kRing) - 1) & 1u, kSleepNs)) {
                    atomicExch(p.err, 3u);
                    break;
                }
                const int s = s0 + r;
                mbar_expect_tx(full + slot, kStage);
                bulk_g2s(ring + slot * kStage, weights_of(s), kUnit, full + slot);
                bulk_g2s(ring + slot * kStage + kUnit, p.xb + (size_t)(s % p.nb) * kBBytes, kBBytes, full + slot);
                issued = r + 1;
            }
            // let every copy this CTA issued land before it may exit
            for (int r = issued - kRing > 0 ? issued - kRing : 0; r < issued; ++r)
                mbar_wait(full + r % kRing, (uint32_t)(r / kRing) & 1u, 1u << 20);
        }
    } else if (n > 0) {
        // --------------------------- decode / epilogue ---------------------------
        pdl_wait();   // the activation scales are written by the previous kernel
        const int m = threadIdx.x;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float tot[4] = {0.f, 0.f, 0.f, 0.f};
        int sc_prev[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float d_prev = 0.f;
        int last_mma = -1;
        for (int r = 0; r <= n; ++r) {
            int sc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            float d = 0.f;
            // decode stage r into tensor-memory buffer r & 1 (the MMAs of stage r-2,
            // which read it, completed before the epilogue of stage r-2)
            if (r < n) {
                const int slot = r % kRing;
                if (!mbar_wait_sleep(full + slot, (uint32_t)(r / kRing) & 1u, kSleepNs)) {
                    *dec_abort = 1;
                } else {
                    const uint8_t* u = ring + slot * kStage;
                    uint32_t L0, L1;
                    iq4_scale_bytes(lds64(u + kQsBytes + m * 8), L0, L1, d);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        sc[i] = ubyte(L0, i) - 32;
                        sc[4 + i] = ubyte(L1, i) - 32;
                    }
                    const uint32_t abuf = tmem + lane_base + (uint32_t)((r & 1) * 64);
#pragma unroll
                    for (int sb = 0; sb < 8; ++sb) {
                        const uint4 q = lds128(u + sb * (kRows * 16) + m * 16);
                        uint32_t a[8];
                        iq4_i8(q.x, a[0], a[1]);
                        iq4_i8(q.y, a[2], a[3]);
                        iq4_i8(q.z, a[4], a[5]);
                        iq4_i8(q.w, a[6], a[7]);
                        tmem_st8(abuf + (uint32_t)(sb * 8), a);
                    }
                    tmem_wait_st();
                }
            }
            // epilogue of stage r-1
            if (r >= 1 && !*dec_abort) {
                const int rp = r - 1;
                if (!mbar_wait_sleep(mma_done, (uint32_t)rp & 1u, kSleepNs)) {
                    *dec_abort = 1;
                } else {
                    tc_fence_after();
                    const uint32_t dbase = tmem + lane_base + kDCol;
                    int acc[12];
#pragma unroll
                    for (int j = 0; j < 12; ++j) acc[j] = 0;
#pragma unroll
                    for (int sb = 0; sb < 8; sb += 2) {
                        uint32_t v0[16], v1[16];
                        tmem_ld16(dbase + (uint32_t)(sb * 16), v0);
                        tmem_ld16(dbase + (uint32_t)((sb + 1) * 16), v1);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 12; ++j)
                            acc[j] += sc_prev[sb] * (int)v0[j] + sc_prev[sb + 1] * (int)v1[j];
                    }
                    const int b_prev = (s0 + rp) % p.nb;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float v = fmaf((float)acc[3 * t], 65536.f,
                                             fmaf((float)acc[3 * t + 1], 256.f, (float)acc[3 * t + 2])) * d_prev;
                        const float xs = t < p.N ? __ldg(p.xqscale + t * p.nb + b_prev) : 0.f;
                        tot[t] = fmaf(xs, v, tot[t]);
                    }
                    if (threadIdx.x == 0) mbar_arrive(empty + rp % kRing);   // weights decoded, digits consumed
                    const int s = s0 + rp;
                    if ((s + 1) % p.nb == 0 || rp == n - 1) {
                        finish_row(p, s / p.nb, cta, s0, s1, m, tot);
#pragma unroll
                        for (int t = 0; t < 4; ++t) tot[t] = 0.f;
                    }
                }
            }
            // every row of stage r is in tensor memory, every read of the accumulators is done
            tc_fence_before();
            named_bar_sync(1, kDecodeThreads);
            if (*dec_abort) break;
            if (r < n && threadIdx.x == 0) {
                tc_fence_after();
                const uint32_t a0 = tmem + (uint32_t)((r & 1) * 64);
                const uint32_t bsm = smem_u32(ring + (r % kRing) * kStage + kUnit);
#pragma unroll
                for (int sb = 0; sb < 8; ++sb)
                    tc_mma_i8(tmem + kDCol + (uint32_t)(sb * 16), a0 + (uint32_t)(sb * 8),
                              smem_desc_kmajor(bsm + (uint32_t)(sb * 512), 128u, 256u), kIdesc, 0u);
                tc_commit(mma_done);
                last_mma = r;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) sc_prev[i] = sc[i];
            d_prev = d;
        }
        if (*dec_abort) {
            if (threadIdx.x == 0) {
                atomicExch(p.err, 4u);
                if (last_mma >= 0) mbar_wait(mma_done, (uint32_t)last_mma & 1u, 1u << 20);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, kCols);
}

// ------------------------ wide GEMM, scales folded ---------------------------
// Up to NT = 16 or 32 input vectors per weight sweep.  The sub-block scale s
// (ls - 32, 6 bits signed) is folded into the weights: each code c of a
// sub-block becomes A = s * kvalues[c] (|A| <= 4064), written to tensor memory
// as two int8 planes A = 64 H + L (L in [-32, 31], H in [-63, 64]) by a
// byte-permute lookup in a shared table indexed by s.  Per (tile, block) stage
// 16 MMAs (M 128, N 3 NT, K 32): the 8 sub-blocks of each plane accumulate into
// one D region, so the sums arrive already scaled, and per (row, token, digit)
// the epilogue forms 64 SH + SL.  That integer is the one the other paths build
// from per-sub-block sums (sum over k of s kv_k D_k), and the digits and the
// fp16 block scale are combined in fp32 in the same order (65536 d0 + (256 d1 +
// d2)), so a (tile, block) gives the same value here and on the mma.sync GEMV.
//
// Warp roles, each stage handed on by mbarriers so that neighbouring stages
// overlap:
//   warp 0       producer: bulk copies of the stage's weights and activation
//                tiles into a 4-slot ring (slot freed by the MMAs' commit);
//   warp 1       allocates the tensor memory; lane 0 issues the 16 MMAs of a
//                stage once its A buffer is full and the epilogue has read D;
//   warps 2-9    decode: two per lane quarter, each half of the sub-blocks of
//                its 32 rows, into one of two A buffers (2 planes x 8 sub-blocks
//                x 8 columns); the rows' block scales go to a 4-deep stage array;
//   warps 10-    epilogue: NT / 8 per lane quarter, 8 tokens each; D is read
//                into registers and released before the arithmetic.
// Tensor memory: A 2 x 128 columns, D (H, L) x 3 NT columns; one CTA per SM.
//
// What bounds it (CUDA-event and per-stage timestamps, 17408 x 5120, 148 CTAs):
// the tensor pipe.  The 16 MMAs of a 32-token stage (6.3 M int8 MACs) issue in
// about 1.1 us, some 2000 MACs per SM clock, and the epilogue's read-out of D
// and the hand-back add about 0.7 us before the next stage's MMAs; the decode
// of the next stage (1.3 us) overlaps.  Exact sums need the 6 products per
// weight and token (2 planes x 3 digits).
template <int NT>
struct Tcw {
    static constexpr int kB = 8 * 3 * NT * 32;          // B tiles of one block
    static constexpr int kStage = kUnit + kB;
    static constexpr int kRing = 4;
    static constexpr uint32_t kDCol = 256;
    static constexpr uint32_t kIdesc = idesc_i8(128, 3 * NT);
    static constexpr int kEpiWarps = NT / 2;            // 4 lane quarters x NT / 8 token groups
    static constexpr int kWarps = 10 + kEpiWarps;
    static constexpr int kThreads = kWarps * 32;
};
constexpr int kLutBytes = 64 * 2 * 16;                  // [H, L][s + 32][code]: 16-byte rows, 8 bank groups
constexpr int kDStage = 4;                              // block scales of the last 4 stages
constexpr int kXsMax = QB_TCW_TOK * 80;                 // activation scales [N][K / 256] (K <= 20480)
constexpr int kHdrW = 256 + kLutBytes + kDStage * kRows * 4 + kXsMax * 4;
constexpr int kTokW = 8;                                // tokens of one epilogue warp
constexpr uint32_t kSpinW = 1u << 24;                   // try_wait rounds of the MMA / epilogue hand-offs (bounded)

// 8 codes (the nibbles of w, element order of iq4_i8) -> bytes of the two planes
__device__ __forceinline__ void lut16x2(uint32_t w, const uint4& TH, const uint4& TL, uint32_t& h0, uint32_t& h1,
                                        uint32_t& l0, uint32_t& l1) {
    const uint32_t idx = w & 0x77777777u;
    const uint32_t sel = ((w >> 1) & 0x44444444u) | 0x32103210u;
    const uint32_t idxh = idx >> 16, selh = sel >> 16;
    h0 = prmt(prmt(TH.x, TH.y, idx), prmt(TH.z, TH.w, idx), sel);
    h1 = prmt(prmt(TH.x, TH.y, idxh), prmt(TH.z, TH.w, idxh), selh);
    l0 = prmt(prmt(TL.x, TL.y, idx), prmt(TL.z, TL.w, idx), sel);
    l1 = prmt(prmt(TL.x, TL.y, idxh), prmt(TL.z, TL.w, idxh), selh);
}

// row m of tile T complete for tokens tb..tb+7 (token group tg): store them, or
// combine the split tile's per-CTA partials of this group (last arriving CTA, CTA order)
template <int NT>
__device__ void finish_row_w(const TcK& p, int T, int cta, int s0, int s1, int m, int tg, const float (&tot)[kTokW]) {
    const int sg = seg_of_tile(p, T);
    const int row = (T - p.tile0[sg]) * kRows + m;
    const int tb = kTokW * tg;
    auto store = [&](const float (&v)[kTokW]) {
        if (row >= p.rows[sg] || row < p.row_lo || row >= p.row_hi) return;
        float prev[kTokW];
#pragma unroll
        for (int t = 0; t < kTokW; ++t)   // L2 loads: this SM's L1 may hold an older copy of the output
            prev[t] = (tb + t < p.N && p.accumulate) ? __ldcg(p.out[sg] + (size_t)(tb + t) * p.ldo[sg] + row) : 0.f;
#pragma unroll
        for (int t = 0; t < kTokW; ++t)
            if (tb + t < p.N) p.out[sg][(size_t)(tb + t) * p.ldo[sg] + row] = p.accumulate ? prev[t] + v[t] : v[t];
    };
    const int P0 = T * p.nb, P1 = P0 + p.nb;
    if (s0 <= P0 && s1 >= P1) {
        store(tot);
        return;
    }
    const int piece = s0 > P0 ? 0 : 1;
    float4* dst = reinterpret_cast<float4*>(p.partial + (((size_t)cta * 2 + piece) * kRows + m) * NT + tb);
    dst[0] = make_float4(tot[0], tot[1], tot[2], tot[3]);
    dst[1] = make_float4(tot[4], tot[5], tot[6], tot[7]);
    const int c_first = stage_cta(p.S, p.G, P0), c_last = stage_cta(p.S, p.G, P1 - 1);
    unsigned* ctr = p.counters + ((size_t)T * kRows + m) * 4 + tg;
    const unsigned old = atom_add_acq_rel_gpu(ctr, 1u);
    if ((int)old != c_last - c_first) return;
    float sum[kTokW];
#pragma unroll
    for (int t = 0; t < kTokW; ++t) sum[t] = 0.f;
    for (int c = c_first; c <= c_last; ++c) {
        const int pc = cta_s0(p.S, p.G, c) > P0 ? 0 : 1;
        const volatile float* v = p.partial + (((size_t)c * 2 + pc) * kRows + m) * NT + tb;
#pragma unroll
        for (int t = 0; t < kTokW; ++t) sum[t] += v[t];
    }
    store(sum);
    *ctr = 0u;
}

template <int NT>
__global__ void __launch_bounds__(Tcw<NT>::kThreads, 1) qmv_tcw_kernel(TcK p) {
    using C = Tcw<NT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);   // [kRing] producer -> decode / MMA
    uint64_t* empty = full + C::kRing;                    // [kRing] MMA commit -> producer
    uint64_t* a_full = empty + C::kRing;                  // [2] decode -> MMA
    uint64_t* a_free = a_full + 2;                        // [2] MMA commit -> decode
    uint64_t* d_full = a_free + 2;                        // MMA commit -> epilogue
    uint64_t* d_free = d_full + 1;                        // epilogue -> MMA
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(d_free + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    uint8_t* lut = smem + 256;
    float* dstage = reinterpret_cast<float*>(smem + 256 + kLutBytes);   // [kDStage][kRows]
    float* xs_s = dstage + kDStage * kRows;                               // [N][nb] activation scales
    uint8_t* ring = smem + kHdrW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int s0 = cta_s0(p.S, p.G, cta), s1 = cta_s0(p.S, p.G, cta + 1);
    const int n = s1 - s0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::kRing; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(a_full + i, 8);   // the 8 decode warps
            mbar_init(a_free + i, 1);
        }
        mbar_init(d_full, 1);
        mbar_init(d_free, C::kEpiWarps);
        *abort_flag = 0;
        mbar_fence_init();
    }
    // planes of s * kvalues[c] for every s: L = ((A + 32) mod 64) - 32, H = (A - L) / 64
    for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
        const int sv = (i >> 4) - 32, c = i & 15;
        const uint32_t kw = c < 4 ? kIq4I8T0 : c < 8 ? kIq4I8T1 : c < 12 ? kIq4I8T2 : kIq4I8T3;   // kvalues
        const int a = sv * (int)(int8_t)(kw >> (8 * (c & 3)));
        const int l = ((a + 32) & 63) - 32;
        lut[(i >> 4) * 16 + c] = (uint8_t)(int8_t)((a - l) >> 6);
        lut[1024 + (i >> 4) * 16 + c] = (uint8_t)(int8_t)l;
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        if (lane == 0 && n > 0) {
            auto weights_of = [&](int s) -> const uint8_t* {
                const int T = s / p.nb, b = s - T * p.nb;
                const int sg = seg_of_tile(p, T);
                return p.w[sg] + ((size_t)(T - p.tile0[sg]) * p.nb + b) * kUnit;
            };
            const int pre = n < C::kRing ? n : C::kRing;
            for (int r = 0; r < pre; ++r) {
                mbar_expect_tx(full + r, C::kStage);
                bulk_g2s(ring + r * C::kStage, weights_of(s0 + r), kUnit, full + r);
            }
            pdl_wait();   // the activation tiles are written by the previous kernel
            for (int r = 0; r < pre; ++r)
                bulk_g2s(ring + r * C::kStage + kUnit, p.xb + (size_t)((s0 + r) % p.nb) * C::kB, C::kB, full + r);
            int issued = pre;
            for (int r = C::kRing; r < n && !*abort_flag; ++r) {
                const int slot = r % C::kRing;
                if (!mbar_wait_sleep(empty + slot, (uint32_t)((r / C::kRing) - 1) & 1u, kSleepNs)) {
                    atomicExch(p.err, 3u);
                    *abort_flag = 1;
                    break;
                }
                const int s = s0 + r;
                mbar_expect_tx(full + slot, C::kStage);
                bulk_g2s(ring + slot * C::kStage, weights_of(s), kUnit, full + slot);
                bulk_g2s(ring + slot * C::kStage + kUnit, p.xb + (size_t)(s % p.nb) * C::kB, C::kB, full + slot);
                issued = r + 1;
            }
            // no copy may still land in shared memory when the CTA exits
            for (int r = issued - C::kRing > 0 ? issued - C::kRing : 0; r < issued; ++r)
                mbar_wait(full + r % C::kRing, (uint32_t)(r / C::kRing) & 1u, 1u << 20);
        }
    } else if (warp == 1) {
        // -------------------------------- MMA ---------------------------------
        if (lane == 0 && n > 0) {
            int last = -1;
            for (int r = 0; r < n; ++r) {
                // the stage's activation tiles (already landed: the decode warps saw them), its A
                // buffer, and D read out by the epilogue of the stage before.  (No suspend hint on
                // these hand-offs: a waiter resumed late leaves the tensor pipe idle.)
                if (!mbar_wait(full + r % C::kRing, (uint32_t)(r / C::kRing) & 1u, kSpinW) ||
                    !mbar_wait(a_full + (r & 1), (uint32_t)(r >> 1) & 1u, kSpinW) ||
                    (r >= 1 && !mbar_wait(d_free, (uint32_t)(r - 1) & 1u, kSpinW)) || *abort_flag) {
                    atomicExch(p.err, 4u);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = tmem + (uint32_t)((r & 1) * 128);
                const uint32_t bsm = smem_u32(ring + (r % C::kRing) * C::kStage + kUnit);
#pragma unroll
                for (int sb = 0; sb < 8; ++sb) {
                    const uint64_t bd = smem_desc_kmajor(bsm + (uint32_t)(sb * 3 * NT * 32), 128u, 256u);
                    tc_mma_i8(tmem + C::kDCol, a0 + (uint32_t)(sb * 8), bd, C::kIdesc, sb > 0 ? 1u : 0u);
                    tc_mma_i8(tmem + C::kDCol + 3u * NT, a0 + 64u + (uint32_t)(sb * 8), bd, C::kIdesc,
                              sb > 0 ? 1u : 0u);
                }
                tc_commit(d_full);
                tc_commit(a_free + (r & 1));
                tc_commit(empty + r % C::kRing);
                last = r;
            }
            // the tensor memory is freed below: the last MMAs must have completed
            if (last >= 0) mbar_wait(a_free + (last & 1), (uint32_t)(last >> 1) & 1u, 1u << 20);
        }
    } else if (warp < 10) {
        // ------------------------------- decode -------------------------------
        if (n > 0) {
            const int q = warp & 3, h = (warp - 2) >> 2;   // lane quarter (warp % 4), sub-block half
            const int m = q * 32 + lane;
            const uint32_t lane_base = (uint32_t)(q * 32) << 16;
            for (int r = 0; r < n; ++r) {
                const int slot = r % C::kRing;
                if (!mbar_wait_sleep(full + slot, (uint32_t)(r / C::kRing) & 1u, kSleepNs) ||
                    (r >= 2 && !mbar_wait_sleep(a_free + (r & 1), (uint32_t)((r - 2) >> 1) & 1u, kSleepNs)) ||
                    *abort_flag) {
                    atomicExch(p.err, 4u);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint8_t* u = ring + slot * C::kStage;
                uint32_t L0, L1;
                float d;
                iq4_scale_bytes(lds64(u + kQsBytes + m * 8), L0, L1, d);
                if (h == 0) dstage[(r % kDStage) * kRows + m] = d;
                const uint32_t abuf = tmem + lane_base + (uint32_t)((r & 1) * 128);
                const uint32_t Lh = h ? L1 : L0;           // ls of sub-blocks 4h..4h+3
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int sb = 4 * h + k;
                    const uint4 qq = lds128(u + sb * (kRows * 16) + m * 16);
                    const uint8_t* tl = lut + ubyte(Lh, k) * 16;   // (ls - 32) + 32
                    const uint4 TH = lds128(tl), TL = lds128(tl + 1024);
                    uint32_t aH[8], aL[8];
                    lut16x2(qq.x, TH, TL, aH[0], aH[1], aL[0], aL[1]);
                    lut16x2(qq.y, TH, TL, aH[2], aH[3], aL[2], aL[3]);
                    lut16x2(qq.z, TH, TL, aH[4], aH[5], aL[4], aL[5]);
                    lut16x2(qq.w, TH, TL, aH[6], aH[7], aL[6], aL[7]);
                    tmem_st8(abuf + (uint32_t)(sb * 8), aH);
                    tmem_st8(abuf + 64u + (uint32_t)(sb * 8), aL);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + (r & 1));
            }
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        if (n > 0) {
            pdl_wait();   // the output rows (accumulate) and the scales are the previous kernels'
            // this launch's activation scales into shared memory (L2 loads: an older copy may be in L1)
            for (int i = threadIdx.x - 320; i < p.N * p.nb; i += C::kEpiWarps * 32) xs_s[i] = __ldcg(p.xqscale + i);
            named_bar_sync(2, C::kEpiWarps * 32);
            const int q = warp & 3, tg = (warp - 10) >> 2;   // lane quarter (warp % 4), token group
            const int m = q * 32 + lane;
            const uint32_t dbase = tmem + ((uint32_t)(q * 32) << 16) + C::kDCol + (uint32_t)(kTokW * tg);
            float tot[kTokW];
#pragma unroll
            for (int t = 0; t < kTokW; ++t) tot[t] = 0.f;
            // column block b and row tile T of stage s0 + r, stepped instead of divided
            int b = s0 % p.nb, T = s0 / p.nb;
            const float* xs_t = xs_s + (size_t)(kTokW * tg) * p.nb;   // this warp's tokens
            for (int r = 0; r < n; ++r) {
                if (!mbar_wait(d_full, (uint32_t)r & 1u, kSpinW) || *abort_flag) {
                    atomicExch(p.err, 4u);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const float d = dstage[(r % kDStage) * kRows + m];
                uint32_t v[6][kTokW];   // (H, L) x digit 0..2
#pragma unroll
                for (int g = 0; g < 3; ++g) {
                    tmem_ld8(dbase + (uint32_t)(g * NT), v[2 * g]);
                    tmem_ld8(dbase + (uint32_t)(3 * NT + g * NT), v[2 * g + 1]);
                }
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(d_free);   // D may take the next stage's sums
#pragma unroll
                for (int t = 0; t < kTokW; ++t) {
                    const int tok = kTokW * tg + t;
                    float f = (float)(64 * (int)v[4][t] + (int)v[5][t]);
                    f = fmaf((float)(64 * (int)v[2][t] + (int)v[3][t]), 256.f, f);
                    const float val = fmaf((float)(64 * (int)v[0][t] + (int)v[1][t]), 65536.f, f) * d;
                    const float xs = tok < p.N ? xs_t[t * p.nb + b] : 0.f;
                    tot[t] = fmaf(xs, val, tot[t]);
                }
                if (b + 1 == p.nb || r == n - 1) {
                    finish_row_w<NT>(p, T, cta, s0, s1, m, tg, tot);
#pragma unroll
                    for (int t = 0; t < kTokW; ++t) tot[t] = 0.f;
                }
                if (++b == p.nb) {
                    b = 0;
                    ++T;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------- repack ---------------------------------------
// GGUF block_iq4_xs rows -> per (128-row tile, 256-column block): qs as
// [8 sub-blocks][128 rows][16 B], then [128 rows][8 B] scales in the
// [A(4) d(2) Bh(2)] form of qb_iq4.cuh.  Rows past `rows` are zeros.
__global__ void repack_tc_kernel(const uint8_t* __restrict__ src, int rows, int nb, int tiles,
                                 uint8_t* __restrict__ dst) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // (tile, block, row)
    if (i >= (long long)tiles * nb * kRows) return;
    const int m = (int)(i % kRows);
    const long long tb = i / kRows;
    const int b = (int)(tb % nb), T = (int)(tb / nb);
    const int r = T * kRows + m;
    uint8_t* u = dst + (size_t)tb * kUnit;
    if (r >= rows) {
        for (int sb = 0; sb < 8; ++sb)
            for (int j = 0; j < 16; ++j) u[sb * (kRows * 16) + m * 16 + j] = 0;
        for (int j = 0; j < 8; ++j) u[kQsBytes + m * 8 + j] = 0;
        return;
    }
    const uint8_t* blk = src + ((size_t)r * nb + b) * 136;
    for (int sb = 0; sb < 8; ++sb)
        for (int j = 0; j < 16; ++j) u[sb * (kRows * 16) + m * 16 + j] = blk[8 + 16 * sb + j];
    const uint32_t sh = blk[2] | (blk[3] << 8);
    const uint32_t sl = blk[4] | (blk[5] << 8) | (blk[6] << 16) | ((uint32_t)blk[7] << 24);
    uint32_t ls[8];
    for (int ib = 0; ib < 8; ++ib) ls[ib] = ((sl >> (4 * ib)) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
    uint32_t A = 0, Bh = 0;
    for (int k = 0; k < 4; ++k) A |= (ls[k] | ((ls[4 + k] & 3) << 6)) << (8 * k);
    for (int k = 0; k < 4; ++k) Bh |= (ls[4 + k] >> 2) << (4 * k);
    const uint32_t dd = blk[0] | (blk[1] << 8);
    uint8_t* s = u + kQsBytes + m * 8;
    for (int k = 0; k < 4; ++k) s[k] = (uint8_t)(A >> (8 * k));
    s[4] = (uint8_t)dd;
    s[5] = (uint8_t)(dd >> 8);
    s[6] = (uint8_t)Bh;
    s[7] = (uint8_t)(Bh >> 8);
}

}  // namespace

size_t qb_repacked_bytes_tc(int rows, int K) {
    if (K % 256) return 0;
    return (size_t)((rows + kRows - 1) / kRows) * (K / 256) * kUnit;
}

cudaError_t qb_repack_tc(const void* src_dev, int rows, int K, void* dst_dev, cudaStream_t st) {
    if (K % 256 || rows < 1) return cudaErrorInvalidValue;
    const int nb = K / 256, tiles = (rows + kRows - 1) / kRows;
    const long long n = (long long)tiles * nb * kRows;
    repack_tc_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint8_t*)src_dev, rows, nb, tiles,
                                                                    (uint8_t*)dst_dev);
    return cudaGetLastError();
}

int qb_qmv_tc_max_ctas() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms * kCtasPerSm;
}

// partial rows of both kernels: 16 token columns (the N <= 4 kernel uses 4 of them per row slot)
size_t qb_qmv_tc_partial_floats(int max_ctas) { return (size_t)max_ctas * 2 * kRows * QB_TCW_TOK; }

cudaError_t qb_qmv_tc(const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate, int row_lo,
                      int row_hi, const QbQmvWork& work, cudaStream_t st) {
    if (nseg < 1 || nseg > QB_MAX_SEG || N < 1 || N > 4 || K % 256 || !xb.xtc || !xb.xqscale)
        return cudaErrorInvalidValue;
    TcK p = {};
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        p.w[i] = (const uint8_t*)segs[i].w;
        p.out[i] = segs[i].out;
        p.ldo[i] = segs[i].ldo;
        p.rows[i] = segs[i].rows;
        p.tile0[i] = tiles;
        tiles += (segs[i].rows + kRows - 1) / kRows;
    }
    p.tile0[nseg] = tiles;
    if ((long long)tiles * kRows > work.max_tc_rows) return cudaErrorInvalidValue;
    p.nseg = nseg;
    p.nb = K / 256;
    p.N = N;
    const long long S = (long long)tiles * p.nb;
    if (S >= (1ll << 30)) return cudaErrorInvalidValue;
    p.S = (int)S;
    int G = qb_qmv_tc_max_ctas();
    if (G > work.max_tc_ctas) G = work.max_tc_ctas;
    if (G > p.S) G = p.S;
    p.G = G;
    p.xb = xb.xtc;
    p.xqscale = xb.xqscale;
    p.accumulate = accumulate;
    p.row_lo = row_lo;
    p.row_hi = row_hi;
    p.partial = work.tc_partial;
    p.counters = work.tc_counters;
    p.err = work.err;
    const size_t smem = kHdr + (size_t)kRing * kStage;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(qmv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    return qb_launch(qmv_tc_kernel, dim3(G), dim3(kThreads), smem, st, p);
}


cudaError_t qb_qmv_tcw(const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate, int row_lo,
                       int row_hi, const QbQmvWork& work, cudaStream_t st) {
    const bool n16 = N <= QB_TC16_TOK;
    if (nseg < 1 || nseg > QB_MAX_SEG || N < 1 || N > QB_TCW_TOK || K % 256 || N * (K / 256) > kXsMax || !xb.xqscale ||
        (n16 ? !xb.xtc16 : !xb.xtc32))
        return cudaErrorInvalidValue;
    TcK p = {};
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        p.w[i] = (const uint8_t*)segs[i].w;
        p.out[i] = segs[i].out;
        p.ldo[i] = segs[i].ldo;
        p.rows[i] = segs[i].rows;
        p.tile0[i] = tiles;
        tiles += (segs[i].rows + kRows - 1) / kRows;
    }
    p.tile0[nseg] = tiles;
    if ((long long)tiles * kRows > work.max_tc_rows) return cudaErrorInvalidValue;
    p.nseg = nseg;
    p.nb = K / 256;
    p.N = N;
    const long long S = (long long)tiles * p.nb;
    if (S >= (1ll << 30)) return cudaErrorInvalidValue;
    p.S = (int)S;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int G = sms;   // one CTA per SM: each holds all 512 tensor-memory columns
    if (G > work.max_tc_ctas) G = work.max_tc_ctas;
    if (G > p.S) G = p.S;
    p.G = G;
    p.xb = n16 ? xb.xtc16 : xb.xtc32;
    p.xqscale = xb.xqscale;
    p.accumulate = accumulate;
    p.row_lo = row_lo;
    p.row_hi = row_hi;
    p.partial = work.tc_partial;
    p.counters = work.tc_counters;
    p.err = work.err;
    if (n16) {
        const size_t smem = kHdrW + (size_t)Tcw<16>::kRing * Tcw<16>::kStage;
        static bool attr16 = false;
        if (!attr16) {
            cudaError_t e = cudaFuncSetAttribute(qmv_tcw_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem);
            if (e != cudaSuccess) return e;
            attr16 = true;
        }
        return qb_launch(qmv_tcw_kernel<16>, dim3(G), dim3(Tcw<16>::kThreads), smem, st, p);
    }
    const size_t smem = kHdrW + (size_t)Tcw<32>::kRing * Tcw<32>::kStage;
    static bool attr32 = false;
    if (!attr32) {
        cudaError_t e = cudaFuncSetAttribute(qmv_tcw_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr32 = true;
    }
    return qb_launch(qmv_tcw_kernel<32>, dim3(G), dim3(Tcw<32>::kThreads), smem, st, p);
}
