// Non-greedy sampling on the device: repetition penalty, temperature, top-k,
// softmax, top-p and the xorshift64 draw of sampler_sample
// (src/sampler.c:61-162), with the seeded stream of the reference.
//
// Work split:
//  * sample_penalty_kernel: one thread walks the last repeat_last_n history
//    tokens oldest first, as the reference does (a token seen twice is
//    penalised twice);
//  * the greedy branch (temp <= 0 or top_k == 1) is the device argmax
//    (argmax_kernel: first maximum, the reference's `>` scan);
//  * sample_topk_block_kernel: each block sorts its 8192 logits as 64-bit keys
//    (ordered value << 32 | ~index) in shared memory, descending, and keeps the
//    first K (K <= 256): the block's top K, ties to the lower index, as the
//    reference's min-heap keeps the earlier of equal values;
//  * sample_draw_kernel: one block folds the blocks' lists into the global top
//    K (the running top K and the next candidates sorted together in shared
//    memory), then one thread repeats the reference's arithmetic in its
//    order (float divides and subtracts, the exp of each term, the double
//    sum, the float normalisation, the top-p prefix, xorshift64, the draw).
//
// The reference computes each term with glibc's expf; here it is CUDA's
// double exp rounded to float, the correctly rounded value.  The two differ
// by one ulp on about 0.06 % of inputs, which moves a sampled token only when
// the draw falls within an ulp of a cumulative boundary.  Exact ties inside
// the top-K list are ordered by index here; the reference's order for them is
// whatever its qsort leaves.
#include "qb_common.cuh"
#include "qb_kernels.h"

namespace {

constexpr int kSampBlock = 8192;   // keys sorted at once in shared memory (64 KB)
constexpr int kSampThreads = 1024;

__device__ __forceinline__ unsigned long long samp_key(float v, uint32_t i) {
    uint32_t u = v == 0.f ? 0u : __float_as_uint(v);   // -0 ranks with +0 (the reference compares with >)
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (0xFFFFFFFFu - i);
}
__device__ __forceinline__ float samp_val(unsigned long long k) {
    const uint32_t u = (uint32_t)(k >> 32);
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
__device__ __forceinline__ uint32_t samp_id(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)k; }

__device__ __forceinline__ bool samp_greedy(const QbSampDev* sd) { return sd->temp <= 0.f || sd->top_k == 1u; }
__device__ __forceinline__ int samp_k(const QbSampDev* sd, int V) {
    int k = (int)sd->top_k;
    if (k > 256) k = 256;
    if (k > V) k = V;
    return k;
}

// bitonic sort of s[0..kSampBlock), descending, by the whole block
__device__ void sort_desc(unsigned long long* s) {
    for (int k = 2; k <= kSampBlock; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < kSampBlock; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = s[i], b = s[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        s[i] = b;
                        s[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
}

// logits[tid] of the history's last repeat_last_n tokens, oldest first (src/sampler.c:64-76)
__global__ void sample_penalty_kernel(float* logits, int V, const QbSampDev* sd) {
    pdl_wait();
    pdl_trigger();
    const float pen = sd->repeat_penalty;
    if (pen == 1.0f || sd->n_hist == 0) return;
    const uint32_t n = sd->n_hist < sd->repeat_last_n ? sd->n_hist : sd->repeat_last_n;
    const uint32_t m = n < QB_SAMP_HIST ? n : QB_SAMP_HIST;
    for (uint32_t i = 0; i < m; ++i) {
        const uint32_t tid = sd->hist[(sd->n_hist - m + i) % QB_SAMP_HIST];
        if (tid < (uint32_t)V) {
            const float x = logits[tid];
            logits[tid] = x > 0.0f ? __fdiv_rn(x, pen) : __fmul_rn(x, pen);
        }
    }
}

// the block's top K keys, sorted descending, to cand[blockIdx.x][0..K)
__global__ void __launch_bounds__(kSampThreads) sample_topk_block_kernel(const float* logits, int V,
                                                                       const QbSampDev* sd,
                                                                       unsigned long long* cand) {
    extern __shared__ unsigned long long s[];
    pdl_wait();
    pdl_trigger();
    if (samp_greedy(sd)) return;
    const int K = samp_k(sd, V);
    const int base = blockIdx.x * kSampBlock;
    for (int i = threadIdx.x; i < kSampBlock; i += kSampThreads) {
        const int g = base + i;
        s[i] = g < V ? samp_key(logits[g], (uint32_t)g) : 0ull;
    }
    __syncthreads();
    sort_desc(s);
    for (int i = threadIdx.x; i < K; i += kSampThreads) cand[(size_t)blockIdx.x * 256 + i] = s[i];
}

// The blocks' lists folded into the top K (the running top K plus the next
// candidates, sorted, as many times as needed), then the reference's
// arithmetic (src/sampler.c:78-161) by one thread.  The token goes to
// sd->token and to the history; the greedy branch takes the device argmax
// am[0] instead.
__global__ void __launch_bounds__(kSampThreads) sample_draw_kernel(const unsigned long long* cand, int nlists,
                                                                 int V, QbSampDev* sd, const uint32_t* am) {
    extern __shared__ unsigned long long s[];
    __shared__ float prob[256];
    pdl_wait();
    pdl_trigger();
    const int t = threadIdx.x;
    uint32_t tok = 0;
    if (samp_greedy(sd)) {
        tok = am[0];
    } else {
        const int K = samp_k(sd, V);
        const int total = nlists * K;
        const int per = kSampBlock - K;   // new candidates per fold
        for (int c0 = 0; c0 < total || c0 == 0; c0 += per) {
            for (int i = t; i < kSampBlock; i += kSampThreads) {
                if (i < K) {
                    if (c0 == 0) s[i] = 0ull;   // no running top K yet
                } else {
                    const int c = c0 + (i - K);
                    s[i] = c < total ? cand[(size_t)(c / K) * 256 + (c % K)] : 0ull;
                }
            }
            __syncthreads();
            sort_desc(s);
            if (c0 + per >= total) break;
        }
        if (t == 0) {
            const float temp = sd->temp;
            const float max_l = __fdiv_rn(samp_val(s[0]), temp);
            double sum = 0.0;
            for (int i = 0; i < K; ++i) {
                const float a = __fsub_rn(__fdiv_rn(samp_val(s[i]), temp), max_l);
                prob[i] = (float)exp((double)a);
                sum += (double)prob[i];
            }
            const float inv_sum = sum > 0.0 ? (float)(1.0 / sum) : 0.0f;
            for (int i = 0; i < K; ++i) prob[i] = __fmul_rn(prob[i], inv_sum);
            int n_cand = K;
            if (sd->top_p < 1.0f) {
                float cum = 0.0f;
                int last = 0;
                for (int i = 0; i < K; ++i) {
                    cum = __fadd_rn(cum, prob[i]);
                    last = i;
                    if (cum >= sd->top_p) break;
                }
                n_cand = last + 1;
            }
            float total_p = 0.0f;
            for (int i = 0; i < n_cand; ++i) total_p = __fadd_rn(total_p, prob[i]);
            unsigned long long x = sd->rng;   // xorshift64 (src/sampler.c:8-15)
            x ^= x << 13;
            x ^= x >> 7;
            x ^= x << 17;
            sd->rng = x;
            const float r = __fmul_rn(__fdiv_rn((float)(x % 10000000ull), 10000000.0f), total_p);
            float acc = 0.0f;
            tok = samp_id(s[0]);
            for (int i = 0; i < n_cand; ++i) {
                acc = __fadd_rn(acc, prob[i]);
                if (acc >= r) {
                    tok = samp_id(s[i]);
                    break;
                }
            }
        }
    }
    if (t == 0) {
        sd->token = tok;
        sd->hist[sd->n_hist % QB_SAMP_HIST] = tok;
        sd->n_hist += 1;
    }
}

}  // namespace

int qb_sample_lists(int V) { return (V + kSampBlock - 1) / kSampBlock; }

cudaError_t qb_sample(float* logits, int V, QbSampDev* sd, unsigned long long* cand, unsigned long long* keys,
                      uint32_t* am, cudaStream_t st) {
    const int nl = qb_sample_lists(V);
    if (V < 1) return cudaErrorInvalidValue;
    static bool attr = false;
    const size_t smem = kSampBlock * sizeof(unsigned long long);
    if (!attr) {
        cudaError_t e;
        if ((e = cudaFuncSetAttribute(sample_topk_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)))
            return e;
        if ((e = cudaFuncSetAttribute(sample_draw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)))
            return e;
        attr = true;
    }
    cudaError_t e;
    if ((e = qb_launch(sample_penalty_kernel, dim3(1), dim3(1), 0, st, logits, V, (const QbSampDev*)sd))) return e;
    if ((e = qb_argmax_reset(keys, 1, st))) return e;
    if ((e = qb_argmax(logits, V, V, 1, keys, st))) return e;
    if ((e = qb_argmax_to_u32(keys, 1, am, st))) return e;
    if ((e = qb_launch(sample_topk_block_kernel, dim3(nl), dim3(kSampThreads), smem, st, (const float*)logits, V,
                       (const QbSampDev*)sd, cand)))
        return e;
    return qb_launch(sample_draw_kernel, dim3(1), dim3(kSampThreads), smem, st, (const unsigned long long*)cand, nl,
                     V, sd, (const uint32_t*)am);
}
