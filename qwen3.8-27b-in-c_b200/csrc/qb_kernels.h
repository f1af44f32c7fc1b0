// Host-side launchers of the sm_100a kernels (internal interface of libqwenb200).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

struct QbXIn {               // one segment of a GEMV input vector set
    const float* x;          // token t at x + t * ldx
    long long ldx;
    const float* norm_w;     // RMSNorm weight applied first (nullptr: none)
    int len;                 // columns, multiple of 256
};

struct QbQSeg {              // one matrix of a fused GEMV launch
    const void* w;           // repacked weights (qb_repack)
    float* out;
    long long ldo;
    int rows;
};

// Scratch of one GEMV stream: split tile-pair partials, per-pair arrival
// counters (zero between launches), error flag (non-zero after a bounded
// wait gave up).
struct QbQmvWork {
    float* partial;          // [max_warps][2][32][8]
    float* gpartial;         // [max_warps][2][32][8] (per CTA, or per warp without CTA grouping)
    unsigned* counters;      // [max_pairs], zero-initialised
    unsigned* bcounters;     // [max_pairs] per 256-row output block (qb_qmv_ex epilogues), zero-initialised
    unsigned* err;           // [1]
    int max_warps;
    int max_pairs;
    // tcgen05 IQ4_XS path (qb_qmv_tc)
    float* tc_partial;       // [max_tc_ctas][2][128][4]
    unsigned* tc_counters;   // [max_tc_rows][4] (per row, or per row and token group of 8), zero-initialised
    int max_tc_ctas;
    long long max_tc_rows;   // rows of all fused matrices, rounded up to 128-row tiles
};

// Prepared activations of one GEMV input (written by qb_xprep, read by qb_qmv).
struct QbXBuf {
    uint2* xfrag;            // fp16 hi/lo mma B fragments (all formats but IQ4_XS), qb_xbuf_bytes
    float* xscale;           // [QB_MAX_TOK][K/256] power-of-two scale of xfrag
    float* xsum;             // [QB_MAX_TOK][K/32] plain column sums (Q4_K / Q5_K)
    uint2* xq;               // int8 digit mma B fragments (IQ4_XS), qb_xbuf_bytes
    float* xqscale;          // [QB_MAX_TOK][K/256] power-of-two scale of xq and xtc
    uint8_t* xtc;            // int8 digits as tcgen05 B tiles, 4 KB per 256 columns (N <= 4)
    uint8_t* xtc16;          // the same for up to 16 tokens, 12 KB per 256 columns (qb_qmv_tcw, 16 tokens)
    uint8_t* xtc32;          // the same for up to 32 tokens, 24 KB per 256 columns (qb_qmv_tcw, 32 tokens)
    // Wide inputs (N > QB_MAX_TOK, up to QB_WIDE rows) for the 8-row formats (xfrag,
    // xscale, xsum, xq): row r is row r % 8 of chunk r / 8, and chunk c is an input of
    // its own (min(8, N - 8c) rows, the N <= 8 layouts above; qb_xb_chunk).  The
    // fragment arrays of chunk c start c * cs_frag / cs_q elements in; the per-row
    // arrays (xscale, xsum, xqscale) keep row r at row r, so the 16- and 32-token
    // tiles share xqscale with the chunks.
    long long cs_frag, cs_q;
};
// chunk c (rows 8c..8c+7) of a wide input of nb = K / 256 blocks
__host__ __device__ inline QbXBuf qb_xb_chunk(const QbXBuf& xb, int c, int nb) {
    QbXBuf r = xb;
    r.xfrag = xb.xfrag ? xb.xfrag + c * xb.cs_frag : nullptr;
    r.xscale = xb.xscale ? xb.xscale + (long long)c * 8 * nb : nullptr;
    r.xsum = xb.xsum ? xb.xsum + (long long)c * 64 * nb : nullptr;
    r.xq = xb.xq ? xb.xq + c * xb.cs_q : nullptr;
    r.xqscale = xb.xqscale ? xb.xqscale + (long long)c * 8 * nb : nullptr;
    return r;
}
// Independent sequences in one launch of a stateful layer kernel (multi-sequence
// decode): sequence s covers input rows [s * T, s * T + T); its position and
// recurrent-slot words lie `ctrl` 32-bit words after sequence 0's, its state
// (recurrent slots, KV cache) `state` floats after, and its first position is its
// position word plus s * pos_step.  One sequence: {1, B, 0, 0, 0}.  The attention
// kernels also take one long prefill chunk as S groups of T queries over the same
// cache: {S, T, 0, 0, T}.
struct QbSeqs {
    int S, T;
    long long ctrl, state;
    int pos_step;
};
enum { QB_XP_F16 = 1, QB_XP_SUM = 2, QB_XP_I8 = 4, QB_XP_TC = 8, QB_XP_TC16 = 16, QB_XP_TC32 = 32 };   // qb_xprep outputs
#define QB_TC16_TOK 16       // input vectors of one qb_qmv_tc16 launch; xqscale rows it needs
#define QB_TCW_TOK 32        // input vectors of one qb_qmv_tcw launch

// ---- quantised GEMV (qb_quant.cu) ----
size_t qb_repacked_bytes(int type, int rows, int K);
cudaError_t qb_repack(int type, const void* src_dev, int rows, int K, void* dst_dev, cudaStream_t st);
// bytes of xfrag / xq for inputs of up to K columns
size_t qb_xfrag_bytes(int K);
size_t qb_xq_bytes(int K);
size_t qb_xtc_bytes(int K);
size_t qb_xtc16_bytes(int K);
size_t qb_xtc32_bytes(int K);
// which qb_xprep outputs a matrix of this type reads at N input vectors
// (IQ4_XS: the tcgen05 tiles when N <= 4 and tc != 0, else the mma.sync fragments)
int qb_xprep_needs(int type, int N = QB_MAX_TOK, int tc = 0);
cudaError_t qb_xprep(const QbXIn* in, int nseg, int N, float eps, const QbXBuf& xb, int what, cudaStream_t st);
cudaError_t qb_qmv(int type, const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate,
                   int row_lo, int row_hi, const QbQmvWork& work, cudaStream_t st);

// Activation preparation of the next GEMV's input, fused into this GEMV: as
// the last tile pair of a 256-row block of the output finishes, its warp
// writes that block's fragments (one matrix per launch, rows a multiple of
// 256, no row range).
//  * NORM: the output is a residual stream x (usually accumulate = 1); the
//    fragments hold x * norm_w, and ss[t * (rows / 256) + b] the block's sum
//    of squares of x.  The consuming launch applies the RMSNorm scale to its
//    outputs (QbInNorm): W (x / rms * w) = (W (x * w)) / rms.
//  * SWIGLU: the matrix interleaves gate and up tiles (tile 2p = gate rows
//    16p..16p+15, tile 2p+1 = the same up rows, qb_interleave_tiles); the
//    output is h = silu(gate) * up at h[t * ldh + j], and the fragments are h's.
enum { QB_EPI_NONE = 0, QB_EPI_NORM = 1, QB_EPI_SWIGLU = 2 };
struct QbEpi {
    int kind;
    const float* norm_w;     // NORM
    float* ss;               // NORM: [N][rows / 256]
    float* h;                // SWIGLU: [N][ldh]
    long long ldh;
    QbXBuf xb;               // fragments of the next input (not the buffer this launch reads)
    int what;                // QB_XP_* the next input's consumers read
};
// Deferred RMSNorm of this launch's input (prepared by a NORM epilogue):
// out *= 1 / sqrt(sum_b ss[t * (K / 256) + b] / K + eps).
struct QbInNorm {
    const float* ss;
    float eps;
};
// Tensor parallelism of one GEMV launch (one process per GPU; the buffers
// involved and the flags lie in an arena every peer has mapped).  Two modes:
//  * gather: the segments hold this rank's rows; every output value is stored
//    both locally and at the same address of each peer's buffer (dst +
//    delta[i], over NVLink), and the launch ends with a bounded cross-rank
//    barrier, so that when it completes every rank holds all rows;
//  * partial (gather = 0): the matrix holds this rank's share of the input
//    columns; the launch writes its partial sums (all rows, accumulate = 0) as
//    8-byte (value, tag) words to part + (sequence parity) * part_slot, the
//    tag being its sequence number, so no fence or flag is needed;
//    qb_tp_reduce then adds every rank's partials, as their tags arrive, to
//    the output.
#define QB_TP_MAX 8
struct QbTp {
    int rank, world;
    long long delta[QB_TP_MAX - 1];   // peer i (ranks in order, this one skipped): its address - ours
    unsigned* flags;                  // [QB_TP_MAX] in the shared arena, zero-initialised
    unsigned* done;                   // zero-initialised
    unsigned* seq;                    // zero-initialised; counts this rank's TP launches
    int gather;
    void* part;                       // partial mode: 2 slots of (value, tag) words in the shared arena
    long long part_slot;              // words per slot
};
// x[t * ldx + e] += sum over ranks r (in rank order) of rank r's partial sums
// of the last partial-mode launch (e < E, t < N), each read once its tag is
// there (bounded wait).  parts[r] = rank r's part buffer mapped here.
cudaError_t qb_tp_reduce(float* x, long long ldx, int E, int N, const QbTp& tp, const void* const* parts,
                         unsigned* err, cudaStream_t st);
// nseg == 0 is allowed with tp (a rank without rows of this launch still takes part in the barrier)
cudaError_t qb_qmv_ex(int type, const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate,
                      const QbInNorm* in_norm, const QbEpi* epi, const QbTp* tp, const QbQmvWork& work,
                      cudaStream_t st);
// Tile-interleaved copy of two repacked matrices of equal shape (rows % 16 == 0):
// dst tile 2i = tile i of a, dst tile 2i + 1 = tile i of b.  dst holds
// qb_repacked_bytes(type, 2 * rows, K) bytes.
cudaError_t qb_interleave_tiles(int type, const void* a, const void* b, int rows, int K, void* dst, cudaStream_t st);
cudaError_t qb_qmv_work_alloc(QbQmvWork& w, int max_pairs);

// ---- IQ4_XS GEMV on tcgen05 (qb_qmv_tc.cu), N <= 4 ----
size_t qb_repacked_bytes_tc(int rows, int K);
cudaError_t qb_repack_tc(const void* src_dev, int rows, int K, void* dst_dev, cudaStream_t st);
int qb_qmv_tc_max_ctas();
size_t qb_qmv_tc_partial_floats(int max_ctas);
// 9..32 input vectors in one weight sweep, sub-block scales folded into the
// weights (two int8 planes per code): activation tiles from xb.xtc16 (N <= 16)
// or xb.xtc32, scales from xb.xqscale [N][K/256]; one CTA per SM; the same
// value per (tile, block) as the mma.sync GEMV
cudaError_t qb_qmv_tcw(const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate, int row_lo,
                       int row_hi, const QbQmvWork& work, cudaStream_t st);
// segs[i].w are qb_repack_tc layouts
cudaError_t qb_qmv_tc(const QbQSeg* segs, int nseg, int K, int N, const QbXBuf& xb, int accumulate, int row_lo,
                      int row_hi, const QbQmvWork& work, cudaStream_t st);
void qb_qmv_work_free(QbQmvWork& w);
cudaError_t qb_qmv_f32(const float* W, int rows, int K, const float* x, long long ldx, int N, float* out,
                       long long ldo, int accumulate, int row_lo, int row_hi, cudaStream_t st);

// ---- layer kernels (qb_layers.cu) ----
struct QbCtrl;   // device control block (qb_engine.h)

// The stateful kernels take the sequences of a multi-sequence forward (sq: S
// sequences of T rows, S * T == B; nullptr: one sequence of B rows).  qb_embed:
// row b's token is tokens[(b / T) * sq->ctrl + b % T].
cudaError_t qb_embed(int type, const void* tok_embd, int n_embd, const uint32_t* tokens, int B, float* out,
                     long long ldo, cudaStream_t st, const QbSeqs* sq = nullptr);
// conv1d + SiLU of all channels, plus the recurrence gates (beta, decay) per (token, v-head)
cudaError_t qb_gdn_conv(const float* qkv, long long ld_qkv, int conv_dim, int B, const float* conv_w,
                        float* state_slots, size_t slot_stride, const uint32_t* cur_slot, int ckpt,
                        float* out, long long ld_out, const float* beta, const float* alpha, long long ld_ba,
                        const float* dt_bias, const float* ssm_a, int n_v, float2* gates, cudaStream_t st,
                        const QbSeqs* sq = nullptr);
cudaError_t qb_gdn_recur(const float* qkvc, long long ld_qkvc, const float2* gates, int n_k, int n_v, int dk, int B,
                         float eps, float* state_slots, size_t slot_stride, const uint32_t* cur_slot, int ckpt,
                         float* out, long long ld_out, cudaStream_t st, const QbSeqs* sq = nullptr);
cudaError_t qb_gdn_out(const float* o, const float* z, long long ld, const float* norm_w, int n_v, int dv,
                       int B, float eps, float* y, cudaStream_t st);
cudaError_t qb_attn_prep(float* q, long long ldq, const float* kv, long long ldkv, const float* q_norm,
                         const float* k_norm, int n_head, int n_kv, int hd, int rope_half,
                         const float* rope_cos, const float* rope_sin, const uint32_t* pos, int B, float eps,
                         float* k_cache, float* v_cache, cudaStream_t st, const QbSeqs* sq = nullptr);
// attention scratch: part_o [S][n_head][QB_MAX_TOK][qb_attn_max_chunks(n_ctx)][256] floats,
// part_ml [S][n_head][QB_MAX_TOK][qb_attn_max_chunks(n_ctx)] float2 (S sequences)
int qb_attn_max_chunks(int n_ctx);
cudaError_t qb_attn_decode(const float* q, long long ldq, const float* k_cache, const float* v_cache,
                           int n_head, int n_kv, int hd, const uint32_t* pos, int B, int n_ctx, float* out,
                           long long ldo, float* part_o, float2* part_ml, const QbXBuf& xb, int what,
                           cudaStream_t st, const QbSeqs* sq = nullptr);   // also emits the o-projection GEMV input
// SwiGLU / gated RMSNorm fused with the GEMV activation prep of their output
cudaError_t qb_silu_mul_xprep(const float* gate, const float* up, long long ld, int n, int B, float* out,
                              const QbXBuf& xb, int what, cudaStream_t st);
cudaError_t qb_gdn_out_xprep(const float* o, const float* z, long long ld, const float* norm_w, int n_v, int dv,
                             int B, float eps, float* y, const QbXBuf& xb, int what, cudaStream_t st);
cudaError_t qb_silu_mul(const float* gate, const float* up, long long ld, int n, int B, float* out,
                        cudaStream_t st);
cudaError_t qb_argmax_reset(unsigned long long* keys, int B, cudaStream_t st);
// keys[b] = max(keys[b], max over i < n of (x[b * ldx + i], index i0 + i)), first index on ties
cudaError_t qb_argmax(const float* x, long long ldx, int n, int B, unsigned long long* keys,
                      cudaStream_t st, int i0 = 0);
cudaError_t qb_argmax_to_u32(const unsigned long long* keys, int B, uint32_t* out, cudaStream_t st);

// Tensor-parallel argmax over a vocabulary split by rows: every rank holds the
// keys of its own rows (qb_argmax with i0 = its first row); qb_tp_argmax stores
// them into every rank's exchange array, waits (bounded) for all ranks' keys of
// the same exchange and writes the index of the largest to out[b] on every rank.
struct QbArgX {
    int rank, world;
    unsigned long long* xk;         // this rank's array [2][QB_TP_MAX][QB_MAX_TOK][2] words (shared arena)
    long long delta[QB_TP_MAX];     // rank r's array address - ours (0 for this rank)
    unsigned* xseq;                 // zero-initialised; counts this rank's exchanges
    unsigned* err;                  // set to 4 when a wait ran out
};
cudaError_t qb_tp_argmax(const unsigned long long* keys, int B, uint32_t* out, const QbArgX& x, cudaStream_t st);
// dst[i] = src[r][i] for i in [r0[r], r1[r]) and every rank r != rank (NVLink loads)
cudaError_t qb_tp_pull_rows(float* dst, const float* const* src, const int* r0, const int* r1, int world, int rank,
                            cudaStream_t st);

// element-wise ops behind the kernels.h host-pointer API
cudaError_t qb_op_rmsnorm(float* out, const float* x, const float* w, long long n, float eps,
                          cudaStream_t st);
cudaError_t qb_op_l2norm(float* out, const float* x, long long n, float eps, cudaStream_t st);
cudaError_t qb_op_act(int which, float* x, long long n, cudaStream_t st);   // 0 silu 1 sigmoid 2 softplus
cudaError_t qb_op_softmax(float* x, long long n, cudaStream_t st);

// ---- non-greedy sampling (qb_sample.cu; src/sampler.c:61-162) ----
#define QB_SAMP_HIST 64   // history ring: the reference penalises at most the last 64 tokens
struct QbSampDev {
    float temp, top_p;
    uint32_t top_k;
    float repeat_penalty;
    uint32_t repeat_last_n;
    uint32_t n_hist;                 // tokens appended so far (the ring holds the last QB_SAMP_HIST)
    unsigned long long rng;          // xorshift64 state
    uint32_t hist[QB_SAMP_HIST];
    uint32_t token;                  // the last sampled token
};
// blocks of the top-K pass over a vocabulary of V (candidate lists of 256 keys each)
int qb_sample_lists(int V);
// Samples from logits[0..V) (penalised in place) with the parameters, history
// and generator in sd; the token lands in sd->token and the history.  cand:
// qb_sample_lists(V) x 256 keys; keys / am: one argmax key and index.
cudaError_t qb_sample(float* logits, int V, QbSampDev* sd, unsigned long long* cand, unsigned long long* keys,
                      uint32_t* am, cudaStream_t st);
