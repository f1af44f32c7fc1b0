// Per-layer kernels of the hybrid decoder (everything except the weight GEMVs).
//
// Reference (all under src/): embedding dequant quant.c:86-182 / model.c:981-983,
// Gated DeltaNet model.c:494-595 (recurrence) and 845-941 (conv1d, norms,
// gating), gated attention model.c:318-406 (RoPE, heads) and 760-811 (Q/K
// norm, KV append), SwiGLU model.c:830-836, greedy argmax model.c:746-756.
//
// Element-wise arithmetic follows the reference order where that is cheap:
// the AVX2 polynomial exp (kernels.c:807-822) is restated exactly, products
// that the reference rounds separately (ISO C, no FP contraction) use the
// _rn intrinsics, and the Gated DeltaNet row dots reproduce the 8-lane
// accumulation + horizontal-sum tree of the AVX2 code.  Scalar libm calls
// (expf / log1pf in the gates and the softmax tail) are evaluated in double
// and rounded once.
#include "qb_common.cuh"
#include "qb_kernels.h"
#include "qb_xprep.cuh"
#include "qb_refmath.cuh"

namespace {

constexpr int kNSlot = 4;   // recurrent-state slots (rollback targets)

__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log1pf_cr(float x) { return (float)log1p((double)x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// horizontal sum of 8 lanes in the AVX2 hsum256 order ((0+4)+(1+5))+((2+6)+(3+7))
__device__ __forceinline__ float hsum8(float v) {
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    return v;
}

// ----------------------------- embedding ------------------------------------
__device__ __forceinline__ float f16bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

__device__ float dequant_elem(int type, const uint8_t* row, int e) {
    switch (type) {
    case QB_F32: return reinterpret_cast<const float*>(row)[e];
    case QB_Q8_0: {
        const uint8_t* b = row + (e >> 5) * 34;
        return __fmul_rn(f16bits(ld16(b)), (float)(int8_t)b[2 + (e & 31)]);
    }
    case QB_IQ4_XS: {
        const uint8_t* b = row + (e >> 8) * 136;
        const int ib = (e & 255) >> 5, j = e & 31;
        const int ls = ((b[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((ld16(b + 2) >> (2 * ib)) & 3) << 4);
        const float dl = __fmul_rn(f16bits(ld16(b)), (float)(ls - 32));
        const uint8_t q = b[8 + ib * 16 + (j & 15)];
        const int nib = j < 16 ? (q & 0xF) : (q >> 4);
        const int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
        return __fmul_rn(dl, (float)kv[nib]);
    }
    case QB_Q6_K: {
        const uint8_t* b = row + (e >> 8) * 210;
        const int i = e & 255, n = i >> 7, r = i & 127, m = r >> 5, l = r & 31;
        const int lo = (b[64 * n + 32 * (m & 1) + l] >> (4 * (m >> 1))) & 0xF;
        const int hi = (b[128 + 32 * n + l] >> (2 * m)) & 3;
        const int q = (lo | (hi << 4)) - 32;
        const int sc = (int8_t)b[192 + 8 * n + (l >> 4) + 2 * m];
        return __fmul_rn(__fmul_rn(f16bits(ld16(b + 208)), (float)sc), (float)q);
    }
    case QB_Q4_K:
    case QB_Q5_K: {
        const bool q5 = type == QB_Q5_K;
        const uint8_t* b = row + (e >> 8) * (q5 ? 176 : 144);
        const int i = e & 255, j = i >> 6, half = (i >> 5) & 1, l = i & 31;
        const int is = 2 * j + half;
        const uint8_t* s = b + 4;
        int sc, m;
        if (is < 4) { sc = s[is] & 63; m = s[is + 4] & 63; }
        else { sc = (s[is + 4] & 0xF) | ((s[is - 4] >> 6) << 4); m = (s[is + 4] >> 4) | ((s[is] >> 6) << 4); }
        const float d1 = __fmul_rn(f16bits(ld16(b)), (float)sc);
        const float m1 = __fmul_rn(f16bits(ld16(b + 2)), (float)m);
        const uint8_t* qs = b + (q5 ? 48 : 16) + 32 * j;
        int q = half ? (qs[l] >> 4) : (qs[l] & 0xF);
        if (q5) q += (b[16 + l] >> is) & 1 ? 16 : 0;
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    default: return 0.f;
    }
}

__host__ __device__ inline size_t row_bytes_of(int type, int n) {
    switch (type) {
    case QB_F32: return (size_t)n * 4;
    case QB_Q8_0: return (size_t)(n / 32) * 34;
    case QB_IQ4_XS: return (size_t)(n / 256) * 136;
    case QB_Q6_K: return (size_t)(n / 256) * 210;
    case QB_Q4_K: return (size_t)(n / 256) * 144;
    case QB_Q5_K: return (size_t)(n / 256) * 176;
    default: return 0;
    }
}

// row b's token: tok[(b / T) * tstride + b % T] (T rows per sequence, each
// sequence's tokens tstride words apart)
__global__ void embed_kernel(int type, const uint8_t* __restrict__ E, int n, const uint32_t* __restrict__ tok,
                             int T, long long tstride, float* __restrict__ out, long long ldo) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const uint8_t* row = E + (size_t)tok[(size_t)(b / T) * tstride + b % T] * row_bytes_of(type, n);
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x)
        out[(size_t)b * ldo + e] = dequant_elem(type, row, e);
}

// ------------------------------ GDN conv ------------------------------------
// conv1d k=4 over the B tokens, state [c][4] newest last (src/model.c:891-903),
// checkpoints per token (904-907), then SiLU (909).
__global__ void gdn_conv_kernel(const float* __restrict__ qkv, long long ld_qkv, int conv_dim, int B,
                                const float* __restrict__ w, float* __restrict__ slots, size_t slot_stride,
                                const uint32_t* __restrict__ cur_slot, int ckpt, float* __restrict__ out,
                                long long ld_out, const float* __restrict__ beta, const float* __restrict__ alpha,
                                long long ld_ba, const float* __restrict__ dt_bias, const float* __restrict__ ssm_a,
                                int n_v, float2* __restrict__ gates, QbSeqs sq) {
    pdl_wait();
    pdl_trigger();
    {   // sequence blockIdx.y: its B rows, its slots and slot index
        const int sidx = blockIdx.y;
        const size_t r0 = (size_t)sidx * B;
        qkv += r0 * ld_qkv;
        out += r0 * ld_out;
        beta += r0 * ld_ba;
        alpha += r0 * ld_ba;
        gates += r0 * n_v;
        slots += (size_t)sidx * sq.state;
        cur_slot += (size_t)sidx * sq.ctrl;
    }
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < n_v * B) {
        // per (token, v-head) gates of the recurrence (src/model.c:494-500):
        // beta = 1/(1+e^-b), decay = e^(A * softplus(a + dt_bias)), softplus = x > 30 ? x : log1p(e^x)
        const int b = c / n_v, h = c - b * n_v;
        const float bs = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-beta[(size_t)b * ld_ba + h])));
        const float a_raw = __fadd_rn(alpha[(size_t)b * ld_ba + h], dt_bias[h]);
        const float a_sp = a_raw > 30.0f ? a_raw : log1pf_cr(expf_cr(a_raw));
        gates[c] = make_float2(bs, expf_cr(__fmul_rn(ssm_a[h], a_sp)));
    }
    if (c >= conv_dim) return;
    const int cur = (int)*cur_slot;
    const float4 s0 = *reinterpret_cast<const float4*>(slots + (size_t)cur * slot_stride + (size_t)c * 4);
    const float4 wv = *reinterpret_cast<const float4*>(w + (size_t)c * 4);
    float s[4] = {s0.x, s0.y, s0.z, s0.w};
    for (int b = 0; b < B; ++b) {
        s[0] = s[1];
        s[1] = s[2];
        s[2] = s[3];
        s[3] = qkv[(size_t)b * ld_qkv + c];
        float y = __fmul_rn(s[0], wv.x);
        y = __fadd_rn(y, __fmul_rn(s[1], wv.y));
        y = __fadd_rn(y, __fmul_rn(s[2], wv.z));
        y = __fadd_rn(y, __fmul_rn(s[3], wv.w));
        int slot = -1;
        if (ckpt) {
            if (b < kNSlot - 1 || b == B - 1) slot = b < kNSlot - 1 ? b : kNSlot - 1;
        } else if (b == B - 1) {
            slot = cur;
        }
        if (slot >= 0)
            *reinterpret_cast<float4*>(slots + (size_t)slot * slot_stride + (size_t)c * 4) =
                make_float4(s[0], s[1], s[2], s[3]);
        out[(size_t)b * ld_out + c] = silu_ref(y);
    }
}

// --------------------------- GDN recurrence ---------------------------------
// Grid (n_v, dk/16); block 128 = 4 warps x 4 rows x 8 lanes.  Lane l8 of a row
// owns columns l8 + 8m (m = 0..15): the AVX2 accumulator lane l8 of
// gdn_ssm_head (src/model.c:502-523).  q and k are L2-normalised here
// (src/model.c:911-916, kernels.c:780-805) in the same 8-lane order.
constexpr int kDK = 128;

__global__ void __launch_bounds__(128) gdn_recur_kernel(
    const float* __restrict__ qkvc, long long ld_qkvc, const float2* __restrict__ gates, int n_k, int n_v, int B,
    float eps, float* __restrict__ slots,
    size_t slot_stride, const uint32_t* __restrict__ cur_slot, int ckpt, float* __restrict__ out,
    long long ld_out, QbSeqs sq) {
    pdl_wait();
    pdl_trigger();
    {   // sequence blockIdx.z: its B rows, its slots and slot index
        const int sidx = blockIdx.z;
        const size_t r0 = (size_t)sidx * B;
        qkvc += r0 * ld_qkvc;
        gates += r0 * n_v;
        out += r0 * ld_out;
        slots += (size_t)sidx * sq.state;
        cur_slot += (size_t)sidx * sq.ctrl;
    }
    __shared__ float qn[QB_MAX_TOK][kDK], kn[QB_MAX_TOK][kDK];
    __shared__ float kq_s[QB_MAX_TOK], beta_s[QB_MAX_TOK], decay_s[QB_MAX_TOK];
    const int h = blockIdx.x, kh = h % n_k;
    const int tid = threadIdx.x, lane = tid & 31, l8 = lane & 7;
    const int grp = tid >> 3;   // 16 groups of 8 lanes
    const int row = blockIdx.y * 16 + grp;
    const int cur = (int)*cur_slot;
    const size_t head_off = (size_t)h * kDK * kDK + (size_t)row * kDK;
    float S[16];
    {
        const float* src = slots + (size_t)cur * slot_stride + head_off;
#pragma unroll
        for (int m = 0; m < 16; ++m) S[m] = src[l8 + 8 * m];
    }
    const float q_scale = __fdiv_rn(1.0f, sqrtf((float)kDK));
    // tokens in groups of QB_MAX_TOK (prefill chunks of up to 32 tokens); the state row
    // stays in registers from one group to the next
    for (int g0 = 0; g0 < B; g0 += QB_MAX_TOK) {
        const int G = min(QB_MAX_TOK, B - g0);
        // this group's state row and its tokens' v values: loads issued first, so that
        // their latency overlaps the q / k norms below
        float vrow[QB_MAX_TOK];
#pragma unroll
        for (int b = 0; b < QB_MAX_TOK; ++b)
            vrow[b] = b < G ? qkvc[(size_t)(g0 + b) * ld_qkvc + (size_t)2 * n_k * kDK + (size_t)h * kDK + row] : 0.f;
        if (g0 > 0) __syncthreads();   // the previous group's qn / kn / gates are consumed

        // L2 norms: group (b, which) for b < G, which in {q, k}.  Every lane of a
        // warp runs the shuffles; inactive groups work on zeros and store nothing.
        for (int base = 0; base < 2 * G; base += 16) {
            const int gi = base + grp;
            const bool act = gi < 2 * G;
            const int b = act ? gi >> 1 : 0, which = gi & 1;
            const float* src = qkvc + (size_t)(g0 + b) * ld_qkvc + (size_t)which * n_k * kDK + (size_t)kh * kDK;
            float acc = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                const float v = act ? src[l8 + 8 * m] : 0.f;
                acc = fmaf(v, v, acc);
            }
            const float ss = hsum8(acc);
            const float nrm = sqrtf(ss);
            const float scale = __fdiv_rn(1.0f, nrm > eps ? nrm : eps);
            if (act) {
                float* dst = which ? kn[b] : qn[b];
#pragma unroll
                for (int m = 0; m < 16; ++m) dst[l8 + 8 * m] = __fmul_rn(src[l8 + 8 * m], scale);
            }
        }
        __syncthreads();
        for (int base = 0; base < G; base += 16) {
            const int b = base + grp;
            const bool act = b < G;
            float acc = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m)
                acc = act ? fmaf(kn[b][l8 + 8 * m], qn[b][l8 + 8 * m], acc) : 0.f;
            const float kq = hsum8(acc);
            if (act && l8 == 0) {
                kq_s[b] = kq;
                const float2 gt = gates[(size_t)(g0 + b) * n_v + h];   // gdn_conv_kernel
                beta_s[b] = gt.x;
                decay_s[b] = gt.y;
            }
        }
        __syncthreads();

#pragma unroll
        for (int b = 0; b < QB_MAX_TOK; ++b) {
            if (b >= G) break;
            float ak = 0.f, aq = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                ak = fmaf(S[m], kn[b][l8 + 8 * m], ak);
                aq = fmaf(S[m], qn[b][l8 + 8 * m], aq);
            }
            const float sk = hsum8(ak), sq = hsum8(aq);
            const float decay = decay_s[b];
            const float v = vrow[b];
            const float delta = __fmul_rn(decay, sk);
            const float dj = __fmul_rn(__fsub_rn(v, delta), beta_s[b]);
            const float o = __fmul_rn(__fadd_rn(__fmul_rn(decay, sq), __fmul_rn(dj, kq_s[b])), q_scale);
#pragma unroll
            for (int m = 0; m < 16; ++m) S[m] = fmaf(dj, kn[b][l8 + 8 * m], __fmul_rn(decay, S[m]));
            const int bt = g0 + b;   // token index in the launch
            if (l8 == 0) out[(size_t)bt * ld_out + (size_t)h * kDK + row] = o;
            int slot = -1;
            if (ckpt) {
                if (bt < kNSlot - 1 || bt == B - 1) slot = bt < kNSlot - 1 ? bt : kNSlot - 1;
            } else if (bt == B - 1) {
                slot = cur;
            }
            if (slot >= 0) {
                float* dst = slots + (size_t)slot * slot_stride + head_off;
#pragma unroll
                for (int m = 0; m < 16; ++m) dst[l8 + 8 * m] = S[m];
            }
        }
    }
}

// per (token, v-head): RMSNorm(o_h, ssm_norm) * SiLU(z_h)  (src/model.c:927-941)
__global__ void gdn_out_kernel(const float* __restrict__ o, const float* __restrict__ z, long long ld,
                               const float* __restrict__ w, int dv, float eps, float* __restrict__ y) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y, h = blockIdx.x;
    const int lane = threadIdx.x;   // 32 lanes, dv = 128: 4 values each, 8-lane chains in lanes 0..7
    const float* oh = o + (size_t)b * ld + (size_t)h * dv;
    const float* zh = z + (size_t)b * ld + (size_t)h * dv;
    // 8-lane accumulation of the AVX2 rmsnorm; lanes 8..31 repeat lanes 0..7
    float acc = 0.f;
    for (int m = 0; m < dv / 8; ++m) {
        const float v = oh[(lane & 7) + 8 * m];
        acc = fmaf(v, v, acc);
    }
    const float ssum = hsum8(acc);
    const float mean = __fdiv_rn(ssum, (float)dv);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
    for (int i = lane; i < dv; i += 32) {
        const float nv = __fmul_rn(__fmul_rn(oh[i], scale), w[i]);
        y[(size_t)b * ld + (size_t)h * dv + i] = __fmul_rn(nv, silu_ref(zh[i]));
    }
}

// The same, fused with the GEMV activation prep of its output (the ssm_out
// input): one warp per pair of 128-wide v-heads = one 256-column block.  The
// norm sums keep gdn_out_kernel's 8-lane chains: lanes 0-7 head 2p, lanes
// 8-15 head 2p+1.
__global__ void __launch_bounds__(128) gdn_out_xprep_kernel(const float* __restrict__ o, const float* __restrict__ z,
                                                            long long ld, const float* __restrict__ w, int n_v,
                                                            float eps, float* __restrict__ y, int N, QbXBuf xb,
                                                            int what) {
    // a GEMV follows: release it before waiting, so that its CTAs take their places and
    // start streaming weights while this short kernel runs
    pdl_trigger();
    pdl_wait();
    constexpr int DV = 128;
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int pb = blockIdx.x * 4 + (threadIdx.x >> 5);   // head pair = block index of the ssm_out input
    const int nb = n_v / 2;
    if (pb >= nb) return;
    const float* ob = o + (size_t)t * ld + (size_t)pb * 2 * DV;
    const float* zb = z + (size_t)t * ld + (size_t)pb * 2 * DV;
    const int hsel = (lane >> 3) & 1;   // 8-lane group -> head of the pair
    float acc = 0.f;
    for (int m = 0; m < DV / 8; ++m) {
        const float v = ob[hsel * DV + (lane & 7) + 8 * m];
        acc = fmaf(v, v, acc);
    }
    const float ssum = hsum8(acc);
    const float mean = __fdiv_rn(ssum, (float)DV);
    const float sc = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
    const float scale[2] = {__shfl_sync(0xffffffffu, sc, 0), __shfl_sync(0xffffffffu, sc, 8)};
    float v[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int d0 = 4 * lane;
        const float4 o4 = *reinterpret_cast<const float4*>(ob + h * DV + d0);
        const float4 z4 = *reinterpret_cast<const float4*>(zb + h * DV + d0);
        const float4 w4 = *reinterpret_cast<const float4*>(w + d0);
        const float ov[4] = {o4.x, o4.y, o4.z, o4.w}, zv[4] = {z4.x, z4.y, z4.z, z4.w}, wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            v[4 * h + k] = __fmul_rn(__fmul_rn(__fmul_rn(ov[k], scale[h]), wv[k]), silu_ref(zv[k]));
        *reinterpret_cast<float4*>(y + (size_t)t * ld + (size_t)pb * 2 * DV + h * DV + d0) =
            make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
    }
    xprep_emit(v, t, pb, N, nb, nb * 256, xb, what, lane);
}

// ----------------------------- attention ------------------------------------
// One warp per (token, head or kv-head).  Lane owns elements lane + 32j.
// q: RMSNorm(q_norm) then RoPE in place; k: RMSNorm(k_norm), append to the
// cache at pos+b, RoPE in the cache; v: append (src/model.c:784-806).
__global__ void attn_prep_kernel(float* __restrict__ q, long long ldq, const float* __restrict__ kv,
                                 long long ldkv, const float* __restrict__ qw, const float* __restrict__ kw,
                                 int n_head, int n_kv, int hd, int half, const float* __restrict__ rc,
                                 const float* __restrict__ rs, const uint32_t* __restrict__ pos0, float eps,
                                 float* __restrict__ kc, float* __restrict__ vc, QbSeqs sq) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;   // input row; sequence b / T, its token b % T
    const int sidx = b / sq.T;
    const int unit = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int nj = hd / 32;   // 8 for hd = 256
    const uint32_t pos = pos0[(size_t)sidx * sq.ctrl] + (uint32_t)(sidx * sq.pos_step) + (uint32_t)(b - sidx * sq.T);
    kc += (size_t)sidx * sq.state;
    vc += (size_t)sidx * sq.state;
    const int kvrow = n_kv * hd;
    if (unit >= n_head + 2 * n_kv) return;
    float v[8];
    if (unit >= n_head + n_kv) {   // V: copy to cache
        const int kh = unit - n_head - n_kv;
        const float* src = kv + (size_t)b * ldkv + kvrow + (size_t)kh * hd;
        float* dst = vc + (size_t)pos * kvrow + (size_t)kh * hd;
        for (int j = 0; j < nj; ++j) dst[lane + 32 * j] = src[lane + 32 * j];
        return;
    }
    const bool is_q = unit < n_head;
    const int hh = is_q ? unit : unit - n_head;
    const float* src = is_q ? q + (size_t)b * ldq + (size_t)hh * 2 * hd : kv + (size_t)b * ldkv + (size_t)hh * hd;
    const float* w = is_q ? qw : kw;
    float ss = 0.f;
    for (int j = 0; j < nj; ++j) {
        v[j] = src[lane + 32 * j];
        ss = fmaf(v[j], v[j], ss);
    }
    ss = warp_sum(ss);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
    for (int j = 0; j < nj; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), w[lane + 32 * j]);
    // RoPE pairs (i, i + half) for i < half (NeoX, partial): half = 32 -> (lane, lane + 32)
    const float* cs = rc + (size_t)pos * half;
    const float* sn = rs + (size_t)pos * half;
    for (int i0 = 0; i0 < half; i0 += 32) {
        const int i = i0 + lane;
        if (i < half) {
            // element i lives in slot i/32, element i+half in slot (i+half)/32 (both on this lane
            // when half is a multiple of 32)
            const int ja = i >> 5, jb = (i + half) >> 5;
            const float v0 = v[ja], v1 = v[jb];
            v[ja] = __fsub_rn(__fmul_rn(v0, cs[i]), __fmul_rn(v1, sn[i]));
            v[jb] = __fadd_rn(__fmul_rn(v0, sn[i]), __fmul_rn(v1, cs[i]));
        }
    }
    float* dst = is_q ? q + (size_t)b * ldq + (size_t)hh * 2 * hd : kc + (size_t)pos * kvrow + (size_t)hh * hd;
    for (int j = 0; j < nj; ++j) dst[lane + 32 * j] = v[j];
}

// Gated GQA attention over the KV cache (src/model.c:353-406, softmax as
// src/kernels.c:901-939), split over position chunks (flash decoding).  The
// G = n_head / n_kv query heads that share a KV head and the B verify tokens
// form NQ = G * B queries; query qi = g * B + b is head kh * G + g of token b
// and attends positions t <= pos + b.
//
// attn_part_kernel: one CTA per (KV head, chunk of kAttnC positions) reads the
// chunk's keys once into shared memory and computes all NQ x kAttnC scores,
// then per query the chunk max m, p_t = exp(s_t - m), l = sum p_t and the
// partial o = sum_t p_t v_t (values read once per CTA).  attn_combine_kernel:
// one CTA per (head, token) merges the chunks: M = max m_c,
// out = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c, times sigmoid(gate).
// The exponentials are the reference's polynomial; the per-chunk rescaling
// makes the result differ from the single-pass reference by rounding only.
constexpr int kAttnC = 32;       // positions per chunk (key and query rows padded by 4 floats in smem)
constexpr int kAttnHD = 256;     // head dimension
constexpr int kAttnMaxQPT = 6;   // queries per thread in the score phase (NQ <= 48)

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}


// QPT = ceil(NQ / 8) queries per thread in the score phase, 2 * QPT in the value phase
template <int QPT>
__global__ void __launch_bounds__(256) attn_part_kernel(const float* __restrict__ q, long long ldq,
                                                        const float* __restrict__ kc, const float* __restrict__ vc,
                                                        int n_head, int n_kv, const uint32_t* __restrict__ pos0p,
                                                        int B, float* __restrict__ part_o,
                                                        float2* __restrict__ part_ml, int max_chunks, QbSeqs sq) {
    pdl_wait();
    pdl_trigger();
    constexpr int HD = kAttnHD, C = kAttnC, KS = HD + 4;   // padded rows: conflict-free 16-byte loads
    const int kh = blockIdx.x, c = blockIdx.y;
    {   // sequence blockIdx.z: its B query rows, KV cache, position and chunk partials
        const int sidx = blockIdx.z;
        q += (size_t)sidx * B * ldq;
        kc += (size_t)sidx * sq.state;
        vc += (size_t)sidx * sq.state;
        pos0p += (size_t)sidx * sq.ctrl;
        const size_t pq = (size_t)sidx * n_head * QB_MAX_TOK * max_chunks;
        part_ml += pq;
        part_o += pq * HD;
    }
    const int pos0 = (int)*pos0p + (int)blockIdx.z * sq.pos_step;
    const int t0 = c * C;
    if (t0 >= pos0 + B) return;
    const int G = n_head / n_kv, NQ = G * B;
    const int nt = min(C, pos0 + B - t0);   // positions of this chunk that exist
    extern __shared__ __align__(16) float sm[];
    float* Ks = sm;              // [C][KS]
    float* Vs = Ks + C * KS;     // [C][HD]
    float* Qs = Vs + C * HD;     // [NQ][KS]
    float* Ss = Qs + NQ * KS;    // [NQ][C] scores, then p
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvrow = n_kv * HD;
    // all copies in flight at once, one wait
    for (int i = tid; i < C * (HD / 4); i += 256) {
        const int t = i / (HD / 4), d4 = i % (HD / 4);
        if (t < nt) {
            const size_t src = (size_t)(t0 + t) * kvrow + (size_t)kh * HD + 4 * d4;
            cp_async16(Ks + t * KS + 4 * d4, kc + src);
            cp_async16(Vs + t * HD + 4 * d4, vc + src);
        } else {
            *reinterpret_cast<float4*>(Ks + t * KS + 4 * d4) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(Vs + t * HD + 4 * d4) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    for (int i = tid; i < NQ * (HD / 4); i += 256) {
        const int qi = i / (HD / 4), d4 = i % (HD / 4);
        const int g = qi / B, b = qi - g * B;
        cp_async16(Qs + qi * KS + 4 * d4, q + (size_t)b * ldq + (size_t)(kh * G + g) * 2 * HD + 4 * d4);
    }
    cp_async_wait_all();
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
    {   // scores: warp w -> positions 4w .. 4w+3; lane -> position 4w + (lane & 3), queries (lane >> 2) + 8j
        const int t = 4 * warp + (lane & 3), qg = lane >> 2;
        float a[QPT];
#pragma unroll
        for (int j = 0; j < QPT; ++j) a[j] = 0.f;
        const float* kr = Ks + t * KS;
        const float* qr = Qs + qg * KS;
#pragma unroll 4
        for (int d4 = 0; d4 < HD / 4; ++d4) {
            const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * d4);
#pragma unroll
            for (int j = 0; j < QPT; ++j) {
                const float4 q4 = *reinterpret_cast<const float4*>(qr + 8 * j * KS + 4 * d4);
                a[j] = fmaf(q4.x, k4.x, a[j]);
                a[j] = fmaf(q4.y, k4.y, a[j]);
                a[j] = fmaf(q4.z, k4.z, a[j]);
                a[j] = fmaf(q4.w, k4.w, a[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < QPT; ++j) {
            const int qi = qg + 8 * j;
            if (qi < NQ) Ss[qi * C + t] = __fmul_rn(a[j], scale);
        }
    }
    __syncthreads();
    // chunk softmax: warp per query, lane -> position
    for (int qi = warp; qi < NQ; qi += 8) {
        const int b = qi % B;
        const int lim = pos0 + b - t0;   // last valid local position
        const float s0 = lane <= lim ? Ss[qi * C + lane] : -INFINITY;
        const float m = warp_max(s0);
        const float p0 = (m != -INFINITY && lane <= lim) ? exp_poly(__fsub_rn(s0, m)) : 0.f;
        Ss[qi * C + lane] = p0;
        const float l = warp_sum(p0);
        if (lane == 0) {
            const int g = qi / B;
            part_ml[((size_t)(kh * G + g) * QB_MAX_TOK + b) * max_chunks + c] = make_float2(m, l);
        }
    }
    __syncthreads();
    {   // o = sum_t p_t v_t: thread -> 4 dims (tid & 63) x queries (tid >> 6) + 4j
        constexpr int QV = 2 * QPT;
        const int d4 = tid & 63, qg = tid >> 6;
        float4 o[QV];
#pragma unroll
        for (int j = 0; j < QV; ++j) o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        const float* pr = Ss + qg * C;
#pragma unroll 2
        for (int t = 0; t < nt; ++t) {
            const float4 v4 = *reinterpret_cast<const float4*>(Vs + t * HD + 4 * d4);
#pragma unroll
            for (int j = 0; j < QV; ++j) {
                const float pt = pr[4 * j * C + t];
                o[j].x = fmaf(pt, v4.x, o[j].x);
                o[j].y = fmaf(pt, v4.y, o[j].y);
                o[j].z = fmaf(pt, v4.z, o[j].z);
                o[j].w = fmaf(pt, v4.w, o[j].w);
            }
        }
#pragma unroll
        for (int j = 0; j < QV; ++j) {
            const int qi = qg + 4 * j;
            if (qi < NQ) {
                const int g = qi / B, b = qi - g * B;
                float* dst = part_o + (((size_t)(kh * G + g) * QB_MAX_TOK + b) * max_chunks + c) * HD + 4 * d4;
                *reinterpret_cast<float4*>(dst) = o[j];
            }
        }
    }
}

__global__ void __launch_bounds__(128) attn_combine_kernel(const float* __restrict__ q, long long ldq,
                                                           const uint32_t* __restrict__ pos0p,
                                                           const float* __restrict__ part_o,
                                                           const float2* __restrict__ part_ml, int max_chunks,
                                                           int n_head, int N, float* __restrict__ out,
                                                           long long ldo, QbXBuf xb, int what, QbSeqs sq) {
    // a GEMV follows: release it before waiting, so that its CTAs take their places and
    // start streaming weights while this short kernel runs
    pdl_trigger();
    pdl_wait();
    constexpr int HD = kAttnHD;
    const int b = blockIdx.y, lane = threadIdx.x & 31;   // input row b: sequence b / T, its token b % T
    const int h = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (h >= n_head) return;
    const int sidx = b / sq.T, tb = b - sidx * sq.T;
    const int nch = ((int)pos0p[(size_t)sidx * sq.ctrl] + sidx * sq.pos_step + tb) / kAttnC + 1;   // chunks up to pos + tb
    const size_t qrow = ((size_t)sidx * n_head + h) * QB_MAX_TOK + tb;
    const float2* ml = part_ml + qrow * max_chunks;
    float M = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, ml[cc].x);
    double L = 0.0;
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};   // dims 4*lane.., 128 + 4*lane..
    const float* po = part_o + qrow * max_chunks * HD + 4 * lane;
    for (int cc = 0; cc < nch; ++cc) {
        const float2 mv = ml[cc];
        const float w = exp_poly(__fsub_rn(mv.x, M));
        L += (double)w * (double)mv.y;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const float4 p4 = *reinterpret_cast<const float4*>(po + (size_t)cc * HD + hh * 128);
            o[4 * hh + 0] = fmaf(w, p4.x, o[4 * hh + 0]);
            o[4 * hh + 1] = fmaf(w, p4.y, o[4 * hh + 1]);
            o[4 * hh + 2] = fmaf(w, p4.z, o[4 * hh + 2]);
            o[4 * hh + 3] = fmaf(w, p4.w, o[4 * hh + 3]);
        }
    }
    const float inv = (float)(1.0 / L);
    const float* gh = q + (size_t)b * ldq + (size_t)h * 2 * HD + HD;
    float v[8];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const float4 g4 = *reinterpret_cast<const float4*>(gh + hh * 128 + 4 * lane);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) v[4 * hh + k] = __fmul_rn(__fmul_rn(o[4 * hh + k], inv), sigmoid_ref(gv[k]));
        *reinterpret_cast<float4*>(out + (size_t)b * ldo + (size_t)h * HD + hh * 128 + 4 * lane) =
            make_float4(v[4 * hh], v[4 * hh + 1], v[4 * hh + 2], v[4 * hh + 3]);
    }
    xprep_emit(v, b, h, N, n_head, n_head * HD, xb, what, lane);
}

__global__ void silu_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up, long long ld,
                                int n, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const size_t o = (size_t)b * ld + i;
        out[o] = __fmul_rn(silu_ref(gate[o]), up[o]);
    }
}

// SwiGLU fused with the GEMV activation prep of its output (the ffn_down
// input): one warp per 256-column block of one token.
__global__ void __launch_bounds__(128) silu_mul_xprep_kernel(const float* __restrict__ gate,
                                                             const float* __restrict__ up, long long ld, int n,
                                                             int N, float* __restrict__ out, QbXBuf xb, int what) {
    // a GEMV follows: release it before waiting, so that its CTAs take their places and
    // start streaming weights while this short kernel runs
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int nb = n >> 8;
    if (b >= nb) return;
    const size_t base = (size_t)t * ld + (size_t)b * 256;
    float v[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const size_t o = base + h * 128 + 4 * lane;
        const float4 g4 = *reinterpret_cast<const float4*>(gate + o);
        const float4 u4 = *reinterpret_cast<const float4*>(up + o);
        v[4 * h + 0] = __fmul_rn(silu_ref(g4.x), u4.x);
        v[4 * h + 1] = __fmul_rn(silu_ref(g4.y), u4.y);
        v[4 * h + 2] = __fmul_rn(silu_ref(g4.z), u4.z);
        v[4 * h + 3] = __fmul_rn(silu_ref(g4.w), u4.w);
        *reinterpret_cast<float4*>(out + o) = make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
    }
    xprep_emit(v, t, b, N, nb, n, xb, what, lane);
}

// ------------------------------- argmax --------------------------------------
// key = ordered(value) << 32 | ~index: the max key is the largest value with
// the lowest index among equals.  This reproduces the reference's scan
// `if (logits[i] > max) ...` seeded with logits[0] (src/model.c:746-756) for
// every input, including the ones a plain ordering gets wrong:
//  - -0 and +0 compare equal there, so both map to the key of +0 and the
//    lower index wins;
//  - a NaN never wins a comparison, so a NaN after index 0 gets the lowest
//    key (it is chosen only if every entry is NaN, and then index 0 wins);
//  - a NaN at index 0 makes every later comparison false, so the scan returns
//    0: that entry gets the highest key.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
    if (v != v) return i == 0 ? ~0ull : (unsigned long long)(0xFFFFFFFFu - i);
    uint32_t u = v == 0.f ? 0u : __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - i);
}

__global__ void argmax_reset_kernel(unsigned long long* keys, int B) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x < B) keys[threadIdx.x] = 0ull;
}

// n < 2^31 entries per row; the loop index is 64-bit so that the last
// stride cannot wrap for n near 2^31.
__global__ void argmax_kernel(const float* __restrict__ x, long long ldx, int n,
                              unsigned long long* __restrict__ keys, int i0) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const float* xr = x + (size_t)b * ldx;
    unsigned long long best = 0ull;
    const long long step = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
        const unsigned long long k = argmax_key(xr[i], (uint32_t)(i0 + i));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(keys + b, best);
}

__global__ void argmax_to_u32_kernel(const unsigned long long* keys, int B, uint32_t* out) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x < B) out[threadIdx.x] = 0xFFFFFFFFu - (uint32_t)(keys[threadIdx.x] & 0xFFFFFFFFull);
}

// Tensor-parallel argmax exchange, one thread per row b.  Exchange s (this
// rank's count + 1) stores the row's key into slot s & 1 of every rank's array
// as two 64-bit words (key half << 32 | s), each stored and loaded whole, so a
// word counts once its low half is s.  A rank starts exchange s + 2, which
// reuses the slot, only after every rank's words of exchange s + 1 arrived,
// which each rank stores only after its exchange s is over.
__global__ void tp_argmax_kernel(const unsigned long long* __restrict__ keys, int B, uint32_t* out, QbArgX x) {
    pdl_wait();
    pdl_trigger();
    const int b = threadIdx.x;
    const unsigned s = *(volatile const unsigned*)x.xseq + 1u;
    __syncthreads();   // every thread has read the count before thread 0 advances it
    if (b < B) {
        const unsigned long long k = keys[b];
        const unsigned long long w0 = (k & 0xFFFFFFFF00000000ull) | s, w1 = (k << 32) | s;
        const size_t at = ((size_t)(s & 1u) * QB_TP_MAX + x.rank) * QB_MAX_TOK + b;
        for (int r = 0; r < x.world; ++r) {
            unsigned long long* d = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(x.xk + 2 * at) +
                                                                          x.delta[r]);
            asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(d), "l"(w0), "l"(w1) : "memory");
        }
        unsigned long long best = 0ull;
        bool ok = true;
        for (int r = 0; r < x.world && ok; ++r) {
            const unsigned long long* src = x.xk + 2 * (((size_t)(s & 1u) * QB_TP_MAX + r) * QB_MAX_TOK + b);
            unsigned long long v0, v1;
            const unsigned long long t0 = global_ns();
            for (uint32_t it = 0;; ++it) {
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v0) : "l"(src) : "memory");
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v1) : "l"(src + 1) : "memory");
                if ((unsigned)v0 == s && (unsigned)v1 == s) break;
                if (peer_wait_over(it, t0, x.err, 4u)) {
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
            const unsigned long long kr = (v0 & 0xFFFFFFFF00000000ull) | (v1 >> 32);
            best = kr > best ? kr : best;
        }
        if (ok) out[b] = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
    }
    __syncthreads();
    if (b == 0) *(volatile unsigned*)x.xseq = s;
}

struct QbPull {
    int world, rank;
    const float* src[QB_TP_MAX];
    int r0[QB_TP_MAX], r1[QB_TP_MAX];
};
// rows [r0[r], r1[r]) of every other rank's copy, by loads over NVLink
__global__ void tp_pull_rows_kernel(float* __restrict__ dst, QbPull p) {
    pdl_wait();
    pdl_trigger();
    for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        const float* src = p.src[r];
        for (int i = p.r0[r] + blockIdx.x * blockDim.x + threadIdx.x; i < p.r1[r]; i += gridDim.x * blockDim.x)
            dst[i] = src[i];
    }
}

// --------------------- kernels.h element-wise ops -----------------------------
__global__ void op_rmsnorm_kernel(float* out, const float* x, const float* w, long long n, float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ float sh[32];
    float ss = 0.f;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += sh[i];
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    __syncthreads();
    for (long long i = threadIdx.x; i < n; i += blockDim.x)
        out[i] = w ? __fmul_rn(__fmul_rn(x[i], scale), w[i]) : __fmul_rn(x[i], scale);
}

__global__ void op_l2norm_kernel(float* out, const float* x, long long n, float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ float sh[32];
    float ss = 0.f;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += sh[i];
    const float nrm = sqrtf(tot);
    const float scale = __fdiv_rn(1.0f, nrm > eps ? nrm : eps);
    __syncthreads();
    for (long long i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(x[i], scale);
}

// silu / sigmoid: vector body via the polynomial exp, scalar tail (n % 8) via
// expf with the reference's clamps (src/kernels.c:825-871); softplus is scalar
// in the reference (874-885).
__global__ void op_act_kernel(int which, float* x, long long n) {
    pdl_wait();
    pdl_trigger();
    const long long body = n & ~7ll;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        float r;
        if (which == 0) {
            if (i < body) r = silu_ref(v);
            else r = v < -20.0f ? __fmul_rn(v, expf_cr(v)) : v > 20.0f ? v : __fdiv_rn(v, __fadd_rn(1.0f, expf_cr(-v)));
        } else if (which == 1) {
            if (i < body) r = sigmoid_ref(v);
            else r = v < -20.0f ? 0.0f : v > 20.0f ? 1.0f : __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-v)));
        } else {
            r = v > 30.0f ? v : v < -30.0f ? expf_cr(v) : log1pf_cr(expf_cr(v));
        }
        x[i] = r;
    }
}

__global__ void op_softmax_kernel(float* x, long long n) {
    pdl_wait();
    pdl_trigger();
    __shared__ float shf[32];
    __shared__ double shd[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float mx = -INFINITY;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, x[i]);
    mx = warp_max(mx);
    if (lane == 0) shf[warp] = mx;
    __syncthreads();
    mx = shf[0];
    for (int i = 1; i < nw; ++i) mx = fmaxf(mx, shf[i]);
    const long long body = n & ~7ll;
    double s = 0.0;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) {
        const float d = __fsub_rn(x[i], mx);
        const float e = i < body ? exp_poly(d) : expf_cr(d);
        x[i] = e;
        s += (double)e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) shd[warp] = s;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < nw; ++i) tot += shd[i];
    const float inv = (float)(1.0 / tot);
    for (long long i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fmul_rn(x[i], inv);
}

}  // namespace

// ================================ launchers ====================================

// the sequences of a multi-sequence launch (sq, S * T == B rows), or one sequence of B rows
static bool seqs_of(const QbSeqs* sq, int B, QbSeqs& out) {
    out = sq ? *sq : QbSeqs{1, B, 0, 0, 0};
    return out.S >= 1 && out.S <= QB_MAX_SEQ && out.T >= 1 && out.S * out.T == B;
}

cudaError_t qb_embed(int type, const void* tok_embd, int n_embd, const uint32_t* tokens, int B, float* out,
                     long long ldo, cudaStream_t st, const QbSeqs* sq) {
    QbSeqs q;
    if (!seqs_of(sq, B, q)) return cudaErrorInvalidValue;
    return qb_launch(embed_kernel, dim3((n_embd + 255) / 256, B), dim3(256), 0, st, type, (const uint8_t*)tok_embd,
                     n_embd, tokens, q.T, q.ctrl, out, ldo);
}

cudaError_t qb_gdn_conv(const float* qkv, long long ld_qkv, int conv_dim, int B, const float* conv_w,
                        float* state_slots, size_t slot_stride, const uint32_t* cur_slot, int ckpt,
                        float* out, long long ld_out, const float* beta, const float* alpha, long long ld_ba,
                        const float* dt_bias, const float* ssm_a, int n_v, float2* gates, cudaStream_t st,
                        const QbSeqs* sq) {
    QbSeqs q;
    if (!seqs_of(sq, B, q)) return cudaErrorInvalidValue;
    const int T = q.T;
    const int threads = conv_dim > n_v * T ? conv_dim : n_v * T;
    return qb_launch(gdn_conv_kernel, dim3((threads + 127) / 128, q.S), dim3(128), 0, st, qkv, ld_qkv, conv_dim, T,
                     conv_w, state_slots, slot_stride, cur_slot, ckpt, out, ld_out, beta, alpha, ld_ba, dt_bias, ssm_a,
                     n_v, gates, q);
}

cudaError_t qb_gdn_recur(const float* qkvc, long long ld_qkvc, const float2* gates, int n_k, int n_v, int dk, int B,
                         float eps, float* state_slots, size_t slot_stride, const uint32_t* cur_slot, int ckpt,
                         float* out, long long ld_out, cudaStream_t st, const QbSeqs* sq) {
    QbSeqs q;
    // more than QB_MAX_TOK tokens per sequence only without checkpoints (prefill chunks)
    if (dk != kDK || !seqs_of(sq, B, q) || (ckpt && q.T > QB_MAX_TOK)) return cudaErrorInvalidValue;
    return qb_launch(gdn_recur_kernel, dim3(n_v, kDK / 16, q.S), dim3(128), 0, st, qkvc, ld_qkvc, gates, n_k, n_v, q.T,
                     eps, state_slots, slot_stride, cur_slot, ckpt, out, ld_out, q);
}

cudaError_t qb_gdn_out(const float* o, const float* z, long long ld, const float* norm_w, int n_v, int dv,
                       int B, float eps, float* y, cudaStream_t st) {
    qb_launch(gdn_out_kernel, dim3(n_v, B), dim3(32), 0, st, o, z, ld, norm_w, dv, eps, y);
    return cudaGetLastError();
}

cudaError_t qb_attn_prep(float* q, long long ldq, const float* kv, long long ldkv, const float* q_norm,
                         const float* k_norm, int n_head, int n_kv, int hd, int rope_half,
                         const float* rope_cos, const float* rope_sin, const uint32_t* pos, int B, float eps,
                         float* k_cache, float* v_cache, cudaStream_t st, const QbSeqs* sq) {
    QbSeqs sqv;
    if (hd != 256 || rope_half % 32 != 0 || rope_half * 2 > hd || !seqs_of(sq, B, sqv)) return cudaErrorInvalidValue;
    const int units = n_head + 2 * n_kv;
    return qb_launch(attn_prep_kernel, dim3((units + 3) / 4, B), dim3(128), 0, st, q, ldq, kv, ldkv, q_norm, k_norm,
                     n_head, n_kv, hd, rope_half, rope_cos, rope_sin, pos, eps, k_cache, v_cache, sqv);
}

int qb_attn_max_chunks(int n_ctx) { return (n_ctx + kAttnC - 1) / kAttnC; }

cudaError_t qb_attn_decode(const float* q, long long ldq, const float* k_cache, const float* v_cache,
                           int n_head, int n_kv, int hd, const uint32_t* pos, int B, int n_ctx, float* out,
                           long long ldo, float* part_o, float2* part_ml, const QbXBuf& xb, int what,
                           cudaStream_t st, const QbSeqs* sq) {
    QbSeqs sqv;
    if (hd != kAttnHD || n_kv < 1 || n_head % n_kv || B < 1 || B > QB_WIDE || !seqs_of(sq, B, sqv) ||
        sqv.T > QB_MAX_TOK)
        return cudaErrorInvalidValue;
    const int N = B;   // rows of all sequences; B from here on: rows per sequence
    B = sqv.T;
    const int G = n_head / n_kv, NQ = G * B;
    if ((NQ + 7) / 8 > kAttnMaxQPT) return cudaErrorInvalidValue;
    const int max_chunks = qb_attn_max_chunks(n_ctx);
    const int qpt = (NQ + 7) / 8;
    // query and score rows up to 8 * qpt are read (rows past NQ hold junk that is never stored)
    const size_t smem = ((size_t)kAttnC * (kAttnHD + 4) + (size_t)kAttnC * kAttnHD + (size_t)8 * qpt * (kAttnHD + 4) +
                         (size_t)8 * qpt * kAttnC) * sizeof(float);
    cudaError_t e = cudaSuccess;
#define QB_ATTN_CASE(Q)                                                                                         \
    case Q: {                                                                                                   \
        static size_t configured_for = 0;                                                                       \
        if (smem > configured_for) {                                                                            \
            if ((e = cudaFuncSetAttribute(attn_part_kernel<Q>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                          (int)smem)) != cudaSuccess)                                           \
                return e;                                                                                       \
            configured_for = smem;                                                                              \
        }                                                                                                       \
        qb_launch(attn_part_kernel<Q>, dim3(n_kv, max_chunks, sqv.S), dim3(256), smem, st, q, ldq, k_cache,     \
                  v_cache, n_head, n_kv, pos, B, part_o, part_ml, max_chunks, sqv);                             \
        break;                                                                                                  \
    }
    switch (qpt) {
        QB_ATTN_CASE(1) QB_ATTN_CASE(2) QB_ATTN_CASE(3) QB_ATTN_CASE(4) QB_ATTN_CASE(5) QB_ATTN_CASE(6)
    default: return cudaErrorInvalidValue;
    }
#undef QB_ATTN_CASE
    return qb_launch(attn_combine_kernel, dim3((n_head + 3) / 4, N), dim3(128), 0, st, q, ldq, pos,
                     (const float*)part_o, (const float2*)part_ml, max_chunks, n_head, N, out, ldo, xb, what, sqv);
}

cudaError_t qb_silu_mul(const float* gate, const float* up, long long ld, int n, int B, float* out,
                        cudaStream_t st) {
    qb_launch(silu_mul_kernel, dim3((n + 255) / 256, B), dim3(256), 0, st, gate, up, ld, n, out);
    return cudaGetLastError();
}

cudaError_t qb_silu_mul_xprep(const float* gate, const float* up, long long ld, int n, int B, float* out,
                              const QbXBuf& xb, int what, cudaStream_t st) {
    if (n % 256 || B < 1 || B > QB_WIDE) return cudaErrorInvalidValue;
    qb_launch(silu_mul_xprep_kernel, dim3((n / 256 + 3) / 4, B), dim3(128), 0, st, gate, up, ld, n, B, out, xb, what);
    return cudaGetLastError();
}

cudaError_t qb_gdn_out_xprep(const float* o, const float* z, long long ld, const float* norm_w, int n_v, int dv,
                             int B, float eps, float* y, const QbXBuf& xb, int what, cudaStream_t st) {
    if (dv != 128 || n_v % 2 || B < 1 || B > QB_WIDE) return cudaErrorInvalidValue;
    qb_launch(gdn_out_xprep_kernel, dim3((n_v / 2 + 3) / 4, B), dim3(128), 0, st, o, z, ld, norm_w, n_v, eps, y, B, xb,
              what);
    return cudaGetLastError();
}

cudaError_t qb_argmax_reset(unsigned long long* keys, int B, cudaStream_t st) {
    return qb_launch(argmax_reset_kernel, dim3(1), dim3(32), 0, st, keys, B);
}

cudaError_t qb_argmax(const float* x, long long ldx, int n, int B, unsigned long long* keys, cudaStream_t st,
                      int i0) {
    if (n < 1) return cudaSuccess;   // no rows here: the keys keep their reset value
    const long long want = ((long long)n + 1023) / 1024;
    const int blocks = want < 148 ? (int)want : 148;
    return qb_launch(argmax_kernel, dim3(blocks, B), dim3(256), 0, st, x, ldx, n, keys, i0);
}

cudaError_t qb_tp_argmax(const unsigned long long* keys, int B, uint32_t* out, const QbArgX& x, cudaStream_t st) {
    if (x.world < 2 || x.world > QB_TP_MAX || x.rank < 0 || x.rank >= x.world || B < 1 || B > QB_MAX_TOK ||
        !x.xk || !x.xseq || !x.err || x.delta[x.rank] != 0)
        return cudaErrorInvalidValue;
    qb_launch(tp_argmax_kernel, dim3(1), dim3(32), 0, st, keys, B, out, x);
    return cudaGetLastError();
}

cudaError_t qb_tp_pull_rows(float* dst, const float* const* src, const int* r0, const int* r1, int world, int rank,
                            cudaStream_t st) {
    if (world < 2 || world > QB_TP_MAX || rank < 0 || rank >= world) return cudaErrorInvalidValue;
    QbPull p = {};
    p.world = world;
    p.rank = rank;
    for (int r = 0; r < world; ++r) {
        if (r != rank && (!src[r] || r0[r] > r1[r])) return cudaErrorInvalidValue;
        p.src[r] = src[r];
        p.r0[r] = r0[r];
        p.r1[r] = r1[r];
    }
    qb_launch(tp_pull_rows_kernel, dim3(148), dim3(256), 0, st, dst, p);
    return cudaGetLastError();
}

cudaError_t qb_argmax_to_u32(const unsigned long long* keys, int B, uint32_t* out, cudaStream_t st) {
    return qb_launch(argmax_to_u32_kernel, dim3(1), dim3(32), 0, st, keys, B, out);
}

cudaError_t qb_op_rmsnorm(float* out, const float* x, const float* w, long long n, float eps, cudaStream_t st) {
    qb_launch(op_rmsnorm_kernel, dim3(1), dim3(1024), 0, st, out, x, w, n, eps);
    return cudaGetLastError();
}
cudaError_t qb_op_l2norm(float* out, const float* x, long long n, float eps, cudaStream_t st) {
    qb_launch(op_l2norm_kernel, dim3(1), dim3(1024), 0, st, out, x, n, eps);
    return cudaGetLastError();
}
cudaError_t qb_op_act(int which, float* x, long long n, cudaStream_t st) {
    const long long blocks = (n + 255) / 256;
    qb_launch(op_act_kernel, dim3((unsigned)(blocks < 4096 ? (blocks ? blocks : 1) : 4096)), dim3(256), 0, st, which, x, n);
    return cudaGetLastError();
}
cudaError_t qb_op_softmax(float* x, long long n, cudaStream_t st) {
    qb_launch(op_softmax_kernel, dim3(1), dim3(1024), 0, st, x, n);
    return cudaGetLastError();
}
