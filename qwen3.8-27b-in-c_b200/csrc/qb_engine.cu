// Device engine + C ABI of libqwenb200.
//
// Forward structure follows the reference engine:
//   model_forward_batch  src/model.c:976-1002   (embed -> 64 layers -> h_save -> norm -> head)
//   gdn_layer_batch      src/model.c:845-974
//   attention_layer_batch src/model.c:760-843
//   mtp_forward(_batch)  src/model.c:1038-1103
//   model_rollback_to    src/model.c:1015-1031
//   spec loop            src/main.c:158-225
// Recurrent states live in 4 device slots per layer; a verify writes the
// state after token b into slot b, and "rollback to b" selects slot b as the
// live state (no copy).  Dynamic values (tokens, positions, live slot, draft
// candidates, accept length) live in a device control block, so whole
// speculative cycles are captured once as CUDA graphs and replayed.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <string>
#include <vector>
#include <mutex>
#include <algorithm>
#include <unordered_map>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "qb_common.cuh"
#include "qb_kernels.h"
#include "qwen_b200.h"

// ------------------------------- errors ---------------------------------------
static thread_local int g_err = 0;
static thread_local char g_err_str[256] = "";

static void set_err(int code, const char* fmt, ...) {
    if (g_err) return;   // keep the first error
    g_err = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err_str, sizeof g_err_str, fmt, ap);
    va_end(ap);
    fprintf(stderr, "libqwenb200: %s\n", g_err_str);
}

#define CK(call)                                                                             \
    do {                                                                                     \
        cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess) {                                                             \
            set_err((int)e_, "%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
            return -1;                                                                       \
        }                                                                                    \
    } while (0)

extern "C" {
double qwen_prof_embed = 0.0, qwen_prof_gdn = 0.0, qwen_prof_attn = 0.0, qwen_prof_head = 0.0;
uint64_t qwen_prof_calls = 0;
}

extern "C" int qb_last_error(void) { return g_err; }
extern "C" const char* qb_last_error_str(void) { return g_err_str; }
extern "C" void qb_clear_error(void) {
    g_err = 0;
    g_err_str[0] = 0;
}

// ----------------------------- GGUF reader ------------------------------------
// Minimal reader of the GGUF v2/v3 container: header, metadata (the
// "<arch>.*" keys of the hybrid model), tensor table, aligned data section.
namespace {

struct GTensor {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    int type = 0;
    uint64_t offset = 0;
    const uint8_t* data = nullptr;
};

struct Gguf {
    int fd = -1;
    size_t size = 0;
    const uint8_t* map = nullptr;
    std::string arch;
    qwen_config_t cfg{};
    std::vector<GTensor> tensors;
    const GTensor* find(const char* n) const {
        for (auto& t : tensors)
            if (t.name == n) return &t;
        return nullptr;
    }
    ~Gguf() {
        if (map) munmap((void*)map, size);
        if (fd >= 0) close(fd);
    }
};

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if ((size_t)(end - p) < sizeof(T)) { ok = false; return v; }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (uint64_t)(end - p)) { ok = false; return {}; }
        std::string s((const char*)p, (size_t)n);
        p += n;
        return s;
    }
    void skip(uint32_t type) {
        static const int fixed[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (type == 8) { (void)str(); return; }
        if (type == 9) {
            const uint32_t et = get<uint32_t>();
            const uint64_t cnt = get<uint64_t>();
            if (et > 12) { ok = false; return; }
            for (uint64_t i = 0; i < cnt && ok; ++i) skip(et);
            return;
        }
        if (type > 12) { ok = false; return; }
        if ((size_t)(end - p) < (size_t)fixed[type]) { ok = false; return; }
        p += fixed[type];
    }
};

// (elements per block, bytes per block) of the formats the engine decodes;
// {0, 0} for any other ggml type id (include/quant.h:14-68, gguf.h:40-64)
struct BlockFmt { uint64_t elems, bytes; };
BlockFmt block_fmt(int type) {
    switch (type) {
    case QB_F32: return {1, 4};
    case QB_Q8_0: return {32, 34};
    case QB_IQ4_XS: return {256, 136};
    case QB_Q6_K: return {256, 210};
    case QB_Q4_K: return {256, 144};
    case QB_Q5_K: return {256, 176};
    default: return {0, 0};
    }
}

// Bytes of a whole tensor, ~0 for a type this engine does not decode (its
// extent is then unknown here; the model checks reject such a tensor where
// the model needs it) or for a size that does not fit 64 bits.
uint64_t gguf_tensor_bytes(int type, const uint64_t* ne, uint32_t n_dims) {
    const BlockFmt f = block_fmt(type);
    if (!f.elems || ne[0] % f.elems) return ~0ull;
    unsigned __int128 b = (unsigned __int128)(ne[0] / f.elems) * f.bytes;
    for (uint32_t d = 1; d < n_dims; ++d) b *= ne[d];
    return b > (unsigned __int128)(~0ull - 1) ? ~0ull : (uint64_t)b;
}

int gguf_load(Gguf& g, const char* path) {
    g.fd = open(path, O_RDONLY);
    if (g.fd < 0) { set_err(-1, "cannot open %s", path); return -1; }
    struct stat st;
    if (fstat(g.fd, &st) != 0 || st.st_size < 24) { set_err(-1, "bad file %s", path); return -1; }
    g.size = (size_t)st.st_size;
    void* m = mmap(nullptr, g.size, PROT_READ, MAP_SHARED, g.fd, 0);
    if (m == MAP_FAILED) { set_err(-1, "mmap failed for %s", path); return -1; }
    g.map = (const uint8_t*)m;
    Cursor c{g.map, g.map + g.size};
    const uint32_t magic = c.get<uint32_t>(), version = c.get<uint32_t>();
    const uint64_t n_t = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (magic != 0x46554747u || version < 2 || version > 3 || n_t == 0 || n_t > 100000) {
        set_err(-1, "%s: not a GGUF v2/v3 file", path);
        return -1;
    }
    uint32_t alignment = 32;
    // pass 1: architecture + alignment; pass 2: "<arch>.*"
    const uint8_t* kv0 = c.p;
    for (int pass = 1; pass <= 2 && c.ok; ++pass) {
        c.p = kv0;
        for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
            const std::string key = c.str();
            const uint32_t t = c.get<uint32_t>();
            if (pass == 1) {
                if (key == "general.architecture" && t == 8) { g.arch = c.str(); continue; }
                if (key == "general.alignment" && t == 4) { const uint32_t a = c.get<uint32_t>(); if (a) alignment = a; continue; }
                c.skip(t);
                continue;
            }
            const std::string pre = g.arch + ".";
            if (key.compare(0, pre.size(), pre) != 0) { c.skip(t); continue; }
            const std::string k = key.substr(pre.size());
            qwen_config_t& f = g.cfg;
            auto u32 = [&](uint32_t& dst) { if (t == 4) dst = c.get<uint32_t>(); else c.skip(t); };
            auto f32 = [&](float& dst) { if (t == 6) dst = c.get<float>(); else c.skip(t); };
            if (k == "embedding_length") u32(f.n_embd);
            else if (k == "attention.head_count") u32(f.n_head);
            else if (k == "attention.head_count_kv") u32(f.n_head_kv);
            else if (k == "attention.key_length") u32(f.head_dim);
            else if (k == "block_count") u32(f.n_layer);
            else if (k == "feed_forward_length") u32(f.n_ff);
            else if (k == "vocab_size") u32(f.vocab_size);
            else if (k == "context_length") u32(f.context_len);
            else if (k == "rope.freq_base") f32(f.rope_theta);
            else if (k == "rope.dimension_count") u32(f.rope_dim_count);
            else if (k == "attention.layer_norm_rms_epsilon") f32(f.rms_norm_eps);
            else if (k == "full_attention_interval") u32(f.full_attn_interval);
            else if (k == "ssm.state_size") u32(f.ssm_state_size);
            else if (k == "ssm.conv_kernel") u32(f.ssm_conv_kernel);
            else if (k == "ssm.inner_size") u32(f.ssm_inner_size);
            else if (k == "ssm.group_count") u32(f.ssm_group_count);
            else if (k == "nextn_predict_layers") u32(f.nextn_layers);
            else if (k == "tie_word_embeddings" && t == 7) f.tie_word_embeddings = c.get<uint8_t>() != 0;
            else if (k == "rope.dimension_sections" && t == 9) {
                const uint32_t et = c.get<uint32_t>();
                const uint64_t cnt = c.get<uint64_t>();
                for (uint64_t j = 0; j < cnt && c.ok; ++j) {
                    if (et == 4 || et == 5) { const uint32_t v = c.get<uint32_t>(); if (j < 4) f.rope_sections[j] = v; }
                    else c.skip(et);
                }
            } else c.skip(t);
        }
        if (pass == 1 && g.arch.empty()) { set_err(-1, "%s: no general.architecture", path); return -1; }
    }
    g.tensors.resize(n_t);
    for (uint64_t i = 0; i < n_t && c.ok; ++i) {
        GTensor& t = g.tensors[i];
        t.name = c.str();
        t.n_dims = c.get<uint32_t>();
        if (t.n_dims > 4) { c.ok = false; break; }
        for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = c.get<uint64_t>();
        t.type = (int)c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
    }
    if (!c.ok) { set_err(-1, "%s: truncated GGUF header", path); return -1; }
    const uint64_t cur = (uint64_t)(c.p - g.map);
    const uint64_t base = (cur + alignment - 1) / alignment * alignment;
    for (auto& t : g.tensors) {
        // the whole tensor must lie inside the file (a truncated file fails
        // here instead of faulting in a later copy)
        const uint64_t bytes = gguf_tensor_bytes(t.type, t.ne, t.n_dims);
        if (base > g.size || t.offset > g.size - base || (bytes != ~0ull && bytes > g.size - base - t.offset)) {
            set_err(-1, "%s: tensor %s extends past the end of the file", path, t.name.c_str());
            return -1;
        }
        t.data = g.map + base + t.offset;
    }
    if (g.cfg.vocab_size == 0) {
        const GTensor* e = g.find("token_embd.weight");
        if (e && e->n_dims == 2) g.cfg.vocab_size = (uint32_t)e->ne[1];
    }
    return 0;
}

size_t gguf_row_bytes(int type, uint64_t ne0) {
    const BlockFmt f = block_fmt(type);
    return f.elems ? ne0 / f.elems * f.bytes : 0;
}

// The structural checks of the reference's model_init (src/model.c:31-53 and
// 55-150: every tensor present, with the dimensions the config implies) plus
// the MTP block blk.<n_layer> (src/model.c:245-279) and the formats this engine
// decodes.  Runs before any device work, so a malformed file makes model_init
// return -1 with a message, as the reference's does.
int validate_model(const Gguf& g) {
    const qwen_config_t& c = g.cfg;
    char nm[96];
    auto find = [&](const char* fmt, int il) -> const GTensor* {
        snprintf(nm, sizeof nm, fmt, il);
        const GTensor* t = g.find(nm);
        if (!t) set_err(-1, "model_init: missing tensor %s", nm);
        return t;
    };
    auto shape = [&](const GTensor* t, uint64_t ne0, uint64_t ne1, bool matrix) -> bool {
        if (!t) return false;
        const bool ok = matrix ? (t->n_dims == 2 && t->ne[0] == ne0 && t->ne[1] == ne1)
                               : (t->n_dims == 1 && t->ne[0] == ne0);
        if (!ok) {
            set_err(-1, "model_init: %s dimension mismatch (%llu x %llu, want %llu x %llu)", t->name.c_str(),
                    (unsigned long long)t->ne[0], (unsigned long long)(t->n_dims > 1 ? t->ne[1] : 1),
                    (unsigned long long)ne0, (unsigned long long)(matrix ? ne1 : 1));
            return false;
        }
        // vectors and the conv1d taps are F32; every other matrix is one of
        // the quantised formats the GEMV decodes
        const BlockFmt f = block_fmt(t->type);
        const bool want_f32 = !matrix || t->name.find("ssm_conv1d") != std::string::npos;
        if (!f.elems || t->ne[0] % f.elems || want_f32 != (t->type == QB_F32)) {
            set_err(-1, "model_init: %s has unsupported type %d for its shape", t->name.c_str(), t->type);
            return false;
        }
        return true;
    };
    if (!c.full_attn_interval || !c.ssm_state_size || !c.n_embd || !c.vocab_size) {
        set_err(-1, "model_init: incomplete model metadata");
        return -1;
    }
    const GTensor* a0 = find("blk.%d.ssm_a", 0);
    if (!a0 || a0->n_dims != 1) { if (a0) set_err(-1, "model_init: blk.0.ssm_a dimension mismatch"); return -1; }
    const uint64_t E = c.n_embd, F = c.n_ff, nv = a0->ne[0], dk = c.ssm_state_size, dv = c.ssm_state_size;
    const uint64_t d_inner = c.ssm_inner_size, conv_dim = 2ull * c.ssm_group_count * dk + d_inner;
    const uint64_t hd = c.head_dim, nh = c.n_head, nkv = c.n_head_kv;
    const uint32_t n_layer = c.n_layer > c.nextn_layers ? c.n_layer - c.nextn_layers : c.n_layer;
    if (d_inner != nv * dv || nv > 256 || dv > 256 || dk > 256) {
        set_err(-1, "model_init: inconsistent DeltaNet sizes (inner %llu, v-heads %llu, state %llu)",
                (unsigned long long)d_inner, (unsigned long long)nv, (unsigned long long)dk);
        return -1;
    }
    const GTensor* te = g.find("token_embd.weight");
    if (!te) { set_err(-1, "model_init: missing tensor token_embd.weight"); return -1; }
    if (!shape(te, E, c.vocab_size, true)) return -1;
    const GTensor* on = g.find("output_norm.weight");
    if (!on) { set_err(-1, "model_init: missing tensor output_norm.weight"); return -1; }
    if (!shape(on, E, 0, false)) return -1;
    const GTensor* out = g.find("output.weight");
    if (out && !shape(out, E, c.vocab_size, true)) return -1;
    auto attn = [&](int il) -> bool {
        return shape(find("blk.%d.attn_q.weight", il), E, 2 * nh * hd, true) &&
               shape(find("blk.%d.attn_k.weight", il), E, nkv * hd, true) &&
               shape(find("blk.%d.attn_v.weight", il), E, nkv * hd, true) &&
               shape(find("blk.%d.attn_output.weight", il), nh * hd, E, true) &&
               shape(find("blk.%d.attn_q_norm.weight", il), hd, 0, false) &&
               shape(find("blk.%d.attn_k_norm.weight", il), hd, 0, false);
    };
    auto common = [&](int il) -> bool {
        return shape(find("blk.%d.attn_norm.weight", il), E, 0, false) &&
               shape(find("blk.%d.post_attention_norm.weight", il), E, 0, false) &&
               shape(find("blk.%d.ffn_gate.weight", il), E, F, true) &&
               shape(find("blk.%d.ffn_up.weight", il), E, F, true) &&
               shape(find("blk.%d.ffn_down.weight", il), F, E, true);
    };
    for (uint32_t il = 0; il < n_layer; ++il) {
        if (!common((int)il)) return -1;
        const bool rec = ((il + 1) % c.full_attn_interval) != 0;
        if (rec) {
            if (!(shape(find("blk.%d.attn_qkv.weight", il), E, conv_dim, true) &&
                  shape(find("blk.%d.attn_gate.weight", il), E, d_inner, true) &&
                  shape(find("blk.%d.ssm_conv1d.weight", il), c.ssm_conv_kernel, conv_dim, true) &&
                  shape(find("blk.%d.ssm_beta.weight", il), E, nv, true) &&
                  shape(find("blk.%d.ssm_alpha.weight", il), E, nv, true) &&
                  shape(find("blk.%d.ssm_out.weight", il), d_inner, E, true) &&
                  shape(find("blk.%d.ssm_dt.bias", il), nv, 0, false) &&
                  shape(find("blk.%d.ssm_a", il), nv, 0, false) &&
                  shape(find("blk.%d.ssm_norm.weight", il), dv, 0, false)))
                return -1;
        } else if (!attn((int)il)) {
            return -1;
        }
    }
    const int im = (int)n_layer;   // the MTP block
    if (!common(im) || !attn(im) || !shape(find("blk.%d.nextn.eh_proj.weight", im), 2 * E, E, true) ||
        !shape(find("blk.%d.nextn.enorm.weight", im), E, 0, false) ||
        !shape(find("blk.%d.nextn.hnorm.weight", im), E, 0, false) ||
        !shape(find("blk.%d.nextn.shared_head_norm.weight", im), E, 0, false))
        return -1;
    return 0;
}

// ------------------------------ engine ----------------------------------------

constexpr int kNSlot = 4;
constexpr int kPrefillW = QB_WIDE;                 // tokens of a wide prefill chunk
constexpr int kAttnGroups = kPrefillW / QB_MAX_TOK;   // its attention query groups

struct DevMat {
    int type = -1;
    int rows = 0, K = 0;
    int row0 = 0, rows_all = 0;   // tensor parallelism: output rows land at row0 + i; rows_all = the tensor's rows
    size_t bytes_all = 0;         // GGUF bytes of the whole tensor (algorithmic traffic of the job)
    void* w = nullptr;      // repacked into 16-row mma.sync tiles (quant) or plain row-major (F32)
    void* w_tc = nullptr;   // IQ4_XS also in 128-row tcgen05 tiles (qb_qmv_tc, N <= 4; qb_qmv_tcw, N > 8)
    const GTensor* src = nullptr;   // the GGUF tensor it came from (whole matrix on one GPU)
    uint64_t fingerprint = 0;   // host-API weight cache only
};

struct LayerW {
    bool rec = false;
    int ridx = -1, aidx = -1;
    const float *attn_norm = nullptr, *post_norm = nullptr;
    DevMat ffn_gate, ffn_up, ffn_down;
    DevMat gu;   // gate and up tiles interleaved (fused SwiGLU epilogue); gate / up keep only their shapes
    DevMat wqkv, wgate, wbeta, walpha, ssm_out;
    const float *conv_w = nullptr, *dt_bias = nullptr, *ssm_a = nullptr, *ssm_norm = nullptr;
    DevMat q, k, v, o;
    const float *q_norm = nullptr, *k_norm = nullptr;
};

}  // namespace

struct QbCtrl {
    uint32_t fwd_pos;
    uint32_t fwd_tok[QB_WIDE];   // up to a 32-token prefill chunk
    uint32_t cur_slot;
    uint32_t mtp_pos;
    uint32_t mtp_tok[QB_WIDE];
    uint32_t argmax[QB_MAX_TOK];
    uint32_t mtp_argmax[QB_MAX_TOK];
    // speculative loop
    uint32_t P, k, cand[QB_MAX_TOK], j, cycle, n_out, next_cand0, n_forced, cap_out, cap_j;
    uint32_t greedy_n;
};

namespace {

struct Engine {
    int dev = 0;
    cudaStream_t st = nullptr;
    Gguf g;
    qwen_config_t cfg{};
    qwen_dims_t d{};
    int V = 0, E = 0, F = 0, n_ctx = 0, rope_half = 0;
    float eps = 1e-6f;
    std::vector<LayerW> L;
    LayerW mtp;
    DevMat eh_proj, output;
    const float *out_norm = nullptr, *enorm = nullptr, *hnorm = nullptr, *shnorm = nullptr;
    int embd_type = 0;
    void* tok_embd = nullptr;   // raw GGUF rows
    std::vector<void*> allocs;

    // state
    float *conv_slots = nullptr, *ssm_slots = nullptr;
    size_t conv_slot_stride = 0, ssm_slot_stride = 0, conv_layer = 0, ssm_layer = 0;
    float *kv_k = nullptr, *kv_v = nullptr, *mtp_k = nullptr, *mtp_v = nullptr;
    size_t kv_layer = 0;
    float *rope_cos = nullptr, *rope_sin = nullptr;

    // activations (QB_WIDE rows each)
    float *bx, *h_save, *qkv, *qkvc, *z, *beta, *alpha, *o, *y, *qbuf, *kvbuf, *attn_o, *gate, *up, *act;
    float *logits, *mtp_x, *mtp_h, *mtp_logits, *emb;
    QbXBuf xb{};                          // prepared GEMV activations (what the next GEMV reads)
    QbXBuf xb_alt{};                      // where a fused GEMV epilogue prepares the input after that
    QbXBuf xb16{};                        // 16-vector tcgen05 activation tiles (qb_bench what = 9)
    const float* xss = nullptr;           // xb holds x * norm_w: per-block sums of squares of x (QbInNorm)
    bool xready = false;                  // xb already holds the next normed input (fused epilogue)
    bool fuse = false;                    // fused GEMV epilogues (QB_FUSE=1; mma.sync path only)
    float* ss = nullptr;                  // [QB_MAX_TOK][Kmax / 256]
    // tensor parallelism (qb_model_init_tp / qb_tp_connect): this rank holds a row
    // range of every quantised matrix; the GEMV outputs live in an arena that every
    // peer maps, and each GEMV stores its rows into all copies
    int tp_rank = 0, tp_world = 1;
    bool tp_ready = false;                // peers connected
    char* arena = nullptr;                // GEMV outputs + TP flags (cudaMalloc'd: IPC-shareable)
    size_t arena_bytes = 0;
    QbTp tp{};
    void* peer_arena[QB_TP_MAX] = {};     // peers' arenas mapped here
    // head-parallel share of this rank (the whole model when tp_world == 1): DeltaNet
    // k-heads [k0, k0 + nk_loc) with their v-heads (local v-head j * nk_loc + i is global
    // j * n_k + k0 + i), attention q-heads [h0, h0 + nh_loc), kv-heads [kv0, kv0 + nkv_loc),
    // FFN columns [f0, f0 + F_loc)
    int nk_loc = 0, nv_loc = 0, nh_loc = 0, nkv_loc = 0, F_loc = 0;
    int k0 = 0, h0 = 0, kv0 = 0, f0 = 0;
    uint2* part = nullptr;                // [2][QB_MAX_TOK][E] (value, tag) partial sums of the residual GEMVs (arena)
    const void* peer_part[QB_TP_MAX] = {};    // rank r's part buffer, mapped here
    QbArgX ax{};                          // argmax exchange of the heads inside the decode graphs
    bool use_tc = false;                  // IQ4_XS at N <= 4 on tcgen05 (QB_TC=1); default: int8 mma.sync
    float* attn_po = nullptr;             // attention chunk partials (qb_attn_decode)
    float2* gates = nullptr;              // DeltaNet (beta, decay) per (token, v-head)
    float2* attn_pml = nullptr;
    unsigned long long* keys = nullptr;   // [2][QB_WIDE]: backbone, mtp
    QbQmvWork work{};
    QbCtrl* ctrl = nullptr;
    uint32_t* d_forced = nullptr;
    uint32_t* d_out_tok = nullptr;
    uint32_t* d_out_j = nullptr;
    uint32_t cap_forced = 0, cap_out = 0, cap_j = 0;
    int ld_qkv = 0;

    // multi-sequence decode (qb_seq_*): n_seq sequences, each with its own recurrent
    // slots, KV caches, control block and MTP hidden row, at these strides (floats) from
    // sequence 0's; the single-sequence paths run on sequence cur_seq
    int n_seq = 1, cur_seq = 0;
    int ms_S = 1;                         // sequences of the forward being recorded (1: single sequence)
    int attn_groups = 1;                  // a 32-token prefill chunk's attention as 4 groups of 8 queries
    long long seq_conv = 0, seq_ssm = 0, seq_kv = 0, seq_mtpkv = 0;
    float *conv_base = nullptr, *ssm_base = nullptr, *kv_k_base = nullptr, *kv_v_base = nullptr;
    float *mtp_k_base = nullptr, *mtp_v_base = nullptr, *mtp_h_base = nullptr;
    QbCtrl* ctrl_base = nullptr;
    uint32_t* wam = nullptr;              // [2][QB_WIDE] argmax of the verify / MTP rows (multi-sequence)
    std::vector<uint32_t> seq_pos;        // tokens consumed per sequence (host)
    cudaGraphExec_t g_mcycle = nullptr;   // one multi-sequence cycle
    int g_mcycle_k = -1;
    size_t mcycle_kernels = 0;

    // graphs
    cudaGraphExec_t g_cycle = nullptr;
    int g_cycle_k = -1;
    size_t cycle_kernels = 0;
    cudaGraphExec_t g_greedy = nullptr;
    cudaGraphExec_t g_sample = nullptr;   // forward + sampling step (qb_sample_generate)
    cudaGraphExec_t g_prefill[2] = {};    // one full prefill chunk, without / with the MTP fill
    cudaGraphExec_t g_prefill_w[2] = {};  // the same for a 32-token chunk
    uint32_t* d_prompt = nullptr;         // [n_ctx] prompt tokens staged for the prefill graphs
    QbSampDev* samp = nullptr;            // sampler parameters, history and generator on the device
    unsigned long long* samp_cand = nullptr;
    unsigned long long* samp_keys = nullptr;
    uint32_t* samp_am = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.f;
    bool any_q45 = false;
    bool tcw = false;                     // IQ4_XS above QB_MAX_TOK rows on qb_qmv_tcw (w_tc of every IQ4_XS matrix)

    ~Engine();
    void* dalloc(size_t bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
        allocs.push_back(p);
        return p;
    }
    void dfree(void* p) {
        for (size_t i = 0; i < allocs.size(); ++i)
            if (allocs[i] == p) {
                cudaFree(p);
                allocs.erase(allocs.begin() + (long)i);
                return;
            }
    }
};

Engine::~Engine() {
    cudaSetDevice(dev);
    for (void*& p : peer_arena)
        if (p) {
            cudaIpcCloseMemHandle(p);
            p = nullptr;
        }
    if (g_cycle) cudaGraphExecDestroy(g_cycle);
    if (g_mcycle) cudaGraphExecDestroy(g_mcycle);
    if (g_greedy) cudaGraphExecDestroy(g_greedy);
    if (g_sample) cudaGraphExecDestroy(g_sample);
    for (cudaGraphExec_t& gp : g_prefill)
        if (gp) cudaGraphExecDestroy(gp);
    for (cudaGraphExec_t& gp : g_prefill_w)
        if (gp) cudaGraphExecDestroy(gp);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    for (void* p : allocs) cudaFree(p);
    qb_qmv_work_free(work);
    if (st) cudaStreamDestroy(st);
}

}  // namespace

// Rows of a matrix held by one rank: whole 32-row tile pairs, split evenly.
extern "C" void qb_tp_rows(int rows, int rank, int world, int* r0, int* r1) {
    const long long pairs = (rows + 31) / 32;
    const int p0 = (int)(pairs * rank / world), p1 = (int)(pairs * (rank + 1) / world);
    *r0 = std::min(rows, 32 * p0);
    *r1 = std::min(rows, 32 * p1);
}

namespace {

// A part of a GGUF matrix to upload: row ranges (start, count) in this order,
// and column ranges of whole quantisation blocks; empty = all.
struct Sel {
    std::vector<std::pair<int, int>> rows, cols;
};

// Gathers the selected rows and column blocks of t into one host buffer in
// GGUF row layout (rows ne0' = the selected columns).  False if a column range
// does not fall on quantisation-block boundaries.
bool gather_host(const GTensor* t, const Sel& sel, std::vector<uint8_t>& out, int& rows, int& cols) {
    const int K = (int)t->ne[0], R = (int)t->ne[1];
    const size_t rb = gguf_row_bytes(t->type, (uint64_t)K);
    const int bc = t->type == QB_F32 ? 1 : t->type == QB_Q8_0 ? 32 : 256;   // columns per block
    const size_t bb = rb / (size_t)(K / bc);                                 // bytes per block
    std::vector<std::pair<int, int>> rr = sel.rows, cc = sel.cols;
    if (rr.empty()) rr.push_back({0, R});
    if (cc.empty()) cc.push_back({0, K});
    rows = cols = 0;
    for (auto& r : rr) rows += r.second;
    for (auto& c : cc) {
        if (c.first % bc || c.second % bc || c.first + c.second > K) return false;
        cols += c.second;
    }
    const size_t orb = (size_t)cols / bc * bb;
    out.resize((size_t)rows * orb);
    uint8_t* o = out.data();
    for (auto& r : rr)
        for (int i = 0; i < r.second; ++i) {
            const uint8_t* row = (const uint8_t*)t->data + (size_t)(r.first + i) * rb;
            for (auto& c : cc) {
                const size_t n = (size_t)c.second / bc * bb;
                memcpy(o, row + (size_t)c.first / bc * bb, n);
                o += n;
            }
        }
    return true;
}

// Uploads the selected part of a quantised matrix, repacked for the GEMV.
// row0 = the global index of its first output row (tensor-parallel gather).
int upload_mat(Engine& e, const GTensor* t, DevMat& m, void* tmp, size_t tmp_bytes, const Sel& sel = Sel(),
               int row0 = 0) {
    if (!t) { set_err(-1, "missing tensor"); return -1; }
    m.type = t->type;
    m.src = t;
    m.rows_all = (int)t->ne[1];
    m.row0 = row0;
    m.bytes_all = gguf_row_bytes(t->type, t->ne[0]) * t->ne[1];
    if (!m.bytes_all || t->type == QB_F32) { set_err(-1, "tensor %s: unsupported type %d", t->name.c_str(), t->type); return -1; }
    std::vector<uint8_t> host;
    const uint8_t* src = (const uint8_t*)t->data;
    size_t src_bytes = m.bytes_all;
    m.K = (int)t->ne[0];
    m.rows = (int)t->ne[1];
    if (!sel.rows.empty() || !sel.cols.empty()) {
        if (!gather_host(t, sel, host, m.rows, m.K)) { set_err(-1, "tensor %s: split off block bounds", t->name.c_str()); return -1; }
        src = host.data();
        src_bytes = host.size();
    }
    if (m.rows == 0) return 0;
    const size_t rb = qb_repacked_bytes(t->type, m.rows, m.K);
    if (!rb || src_bytes > tmp_bytes) { set_err(-1, "tensor %s: cannot repack", t->name.c_str()); return -1; }
    m.w = e.dalloc(rb);
    if (!m.w) { set_err(-2, "cudaMalloc %zu", rb); return -1; }
    // stream-ordered: the repack must not start before the host->device copy lands
    CK(cudaMemcpyAsync(tmp, src, src_bytes, cudaMemcpyHostToDevice, e.st));
    CK(qb_repack(t->type, tmp, m.rows, m.K, m.w, e.st));
    if (t->type == QB_IQ4_XS && e.use_tc) {
        const size_t rt = qb_repacked_bytes_tc(m.rows, m.K);
        m.w_tc = e.dalloc(rt);
        if (!m.w_tc) { set_err(-2, "cudaMalloc %zu", rt); return -1; }
        CK(qb_repack_tc(tmp, m.rows, m.K, m.w_tc, e.st));
    }
    CK(cudaStreamSynchronize(e.st));   // the host buffer must outlive the copy
    if (t->type == QB_Q4_K || t->type == QB_Q5_K) e.any_q45 = true;
    return 0;
}

// Uploads the selected rows of an F32 tensor (a vector is one row of ne0 values,
// selected by columns; a matrix [ne1][ne0] by rows).
const float* upload_f32(Engine& e, const GTensor* t, const Sel& sel = Sel()) {
    if (!t || t->type != QB_F32) return nullptr;
    std::vector<uint8_t> host;
    int rows = 0, cols = 0;
    if (!gather_host(t, sel, host, rows, cols)) return nullptr;
    void* p = e.dalloc(host.size());
    if (!p) return nullptr;
    if (cudaMemcpyAsync(p, host.data(), host.size(), cudaMemcpyHostToDevice, e.st) != cudaSuccess) return nullptr;
    if (cudaStreamSynchronize(e.st) != cudaSuccess) return nullptr;
    return (const float*)p;
}

// gate / up of one FFN as one tile-interleaved matrix for the fused SwiGLU
// epilogue; the separate copies are released (their shapes stay for accounting)
int build_gu(Engine& e, LayerW& l) {
    const DevMat &g = l.ffn_gate, &u = l.ffn_up;
    if (!e.fuse || g.type != u.type || g.type == QB_F32 || g.rows != u.rows || g.K != u.K || g.rows % 256) return 0;
    l.gu.type = g.type;
    l.gu.rows = 2 * g.rows;
    l.gu.K = g.K;
    const size_t rb = qb_repacked_bytes(g.type, l.gu.rows, g.K);
    l.gu.w = e.dalloc(rb);
    if (!l.gu.w) { set_err(-2, "cudaMalloc %zu", rb); return -1; }
    CK(qb_interleave_tiles(g.type, g.w, u.w, g.rows, g.K, l.gu.w, e.st));
    CK(cudaStreamSynchronize(e.st));
    e.dfree(l.ffn_gate.w);
    e.dfree(l.ffn_up.w);
    l.ffn_gate.w = l.ffn_up.w = nullptr;
    return 0;
}

int engine_init(Engine& e, const char* path, uint32_t n_ctx) {
    // host-side parse and checks first: a malformed file fails without device work
    if (gguf_load(e.g, path) || validate_model(e.g)) return -1;
    if (n_ctx == 0) { set_err(-1, "model_init: n_ctx must be > 0"); return -1; }
    CK(cudaGetDevice(&e.dev));
    CK(cudaStreamCreateWithFlags(&e.st, cudaStreamNonBlocking));
    e.cfg = e.g.cfg;
    qwen_config_t& c = e.cfg;
    qwen_dims_t& d = e.d;
    d.n_embd = c.n_embd;
    d.n_ff = c.n_ff;
    d.n_head = c.n_head;
    d.n_kv_head = c.n_head_kv;
    d.head_dim = c.head_dim;
    d.n_k_heads = c.ssm_group_count;
    d.head_k_dim = d.head_v_dim = d.d_state = c.ssm_state_size;
    d.d_inner = c.ssm_inner_size;
    d.d_conv = c.ssm_conv_kernel;
    memcpy(d.rope_sections, c.rope_sections, sizeof d.rope_sections);
    const GTensor* a0 = e.g.find("blk.0.ssm_a");
    if (!a0) { set_err(-1, "missing blk.0.ssm_a"); return -1; }
    d.n_v_heads = (uint32_t)a0->ne[0];
    d.conv_dim = 2 * d.n_k_heads * d.head_k_dim + d.d_inner;
    d.n_layer = c.n_layer > c.nextn_layers ? c.n_layer - c.nextn_layers : c.n_layer;
    if (d.d_inner != d.n_v_heads * d.head_v_dim || d.head_k_dim != 128 || d.head_dim != 256 ||
        d.d_conv != 4 || c.rope_dim_count % 64 != 0 || c.nextn_layers < 1) {
        set_err(-1, "unsupported model shape (head_k_dim %u head_dim %u d_conv %u rope %u)", d.head_k_dim,
                d.head_dim, d.d_conv, c.rope_dim_count);
        return -1;
    }
    e.E = (int)d.n_embd;
    e.F = (int)d.n_ff;
    e.V = (int)c.vocab_size;
    e.eps = c.rms_norm_eps;
    e.n_ctx = (int)n_ctx;
    e.rope_half = (int)c.rope_dim_count / 2;
    {
        // tensor parallelism runs the mma.sync GEMV without fused epilogues
        const char* tc = getenv("QB_TC");
        e.use_tc = e.tp_world == 1 && tc && tc[0] == '1';
        const char* fz = getenv("QB_FUSE");
        e.fuse = e.tp_world == 1 && !e.use_tc && fz && fz[0] == '1';
    }

    // temp buffer for repacking = largest quantised tensor
    size_t tmp_bytes = 0;
    for (auto& t : e.g.tensors)
        if (t.type != QB_F32) tmp_bytes = std::max(tmp_bytes, gguf_row_bytes(t.type, t.ne[0]) * t.ne[1]);
    void* tmp = nullptr;
    CK(cudaMalloc(&tmp, tmp_bytes));
    struct TmpFree { void* p; ~TmpFree() { cudaFree(p); } } tmp_guard{tmp};

    char nm[96];
    auto T = [&](const char* fmt, int il) -> const GTensor* {
        snprintf(nm, sizeof nm, fmt, il);
        const GTensor* t = e.g.find(nm);
        if (!t) set_err(-1, "missing tensor %s", nm);
        return t;
    };
    const GTensor* te = e.g.find("token_embd.weight");
    if (!te || te->ne[0] != (uint64_t)e.E) { set_err(-1, "token_embd missing or wrong shape"); return -1; }
    e.embd_type = te->type;
    {
        const size_t b = gguf_row_bytes(te->type, te->ne[0]) * te->ne[1];
        e.tok_embd = e.dalloc(b);
        if (!e.tok_embd) { set_err(-2, "cudaMalloc token_embd"); return -1; }
        CK(cudaMemcpyAsync(e.tok_embd, te->data, b, cudaMemcpyHostToDevice, e.st));
        CK(cudaStreamSynchronize(e.st));
    }
    // ---- this rank's share (tensor parallelism) ----
    const int g = e.tp_world, rk = e.tp_rank;
    const int nk = (int)d.n_k_heads, nv = (int)d.n_v_heads, nh = (int)d.n_head, nkv = (int)d.n_kv_head;
    const int dk = (int)d.head_k_dim, hd = (int)d.head_dim;
    if (g > 1 && (nk % g || (nk / g) % 2 || nv % nk || nh % g || !(nkv % g == 0 || g % nkv == 0) || e.F % 256 ||
                  (e.F / 256) < g)) {
        set_err(-1, "tensor parallelism over %d ranks needs k-heads / ranks even and q-/kv-heads and FFN "
                    "blocks divisible (k-heads %d, q-heads %d, kv-heads %d, FFN %d)", g, nk, nh, nkv, e.F);
        return -1;
    }
    e.nk_loc = nk / g;
    e.k0 = rk * e.nk_loc;
    e.nv_loc = nv / g;
    e.nh_loc = nh / g;
    e.h0 = rk * e.nh_loc;
    if (nkv % g == 0) {
        e.nkv_loc = nkv / g;
        e.kv0 = rk * e.nkv_loc;
    } else {   // fewer kv-heads than ranks: each rank keeps the one its q-heads use
        e.nkv_loc = 1;
        e.kv0 = e.h0 / (nh / nkv);
    }
    if (g > 1) {   // whole 256-column blocks of the FFN
        const int nb = e.F / 256, b0 = (int)((long long)nb * rk / g), b1 = (int)((long long)nb * (rk + 1) / g);
        e.f0 = b0 * 256;
        e.F_loc = (b1 - b0) * 256;
    } else {
        e.f0 = 0;
        e.F_loc = e.F;
    }
    Sel s_qkv, s_z, s_ba, s_out, s_q, s_kv, s_o, s_up, s_down, s_head;
    int head_row0 = 0;
    if (g > 1) {
        const int R3 = nv / nk;   // v-heads per k-head
        s_qkv.rows.push_back({e.k0 * dk, e.nk_loc * dk});
        s_qkv.rows.push_back({(nk + e.k0) * dk, e.nk_loc * dk});
        for (int j = 0; j < R3; ++j) {
            s_qkv.rows.push_back({2 * nk * dk + (j * nk + e.k0) * dk, e.nk_loc * dk});
            s_z.rows.push_back({(j * nk + e.k0) * dk, e.nk_loc * dk});
            s_ba.rows.push_back({j * nk + e.k0, e.nk_loc});
            s_out.cols.push_back({(j * nk + e.k0) * dk, e.nk_loc * dk});
        }
        s_q.rows.push_back({e.h0 * 2 * hd, e.nh_loc * 2 * hd});
        s_kv.rows.push_back({e.kv0 * hd, e.nkv_loc * hd});
        s_o.cols.push_back({e.h0 * hd, e.nh_loc * hd});
        s_up.rows.push_back({e.f0, e.F_loc});
        s_down.cols.push_back({e.f0, e.F_loc});
    }
    Sel s_vec = s_ba;   // per-v-head vectors: the same heads, as columns of one row
    s_vec.cols = s_ba.rows;
    s_vec.rows.clear();
    Sel s_conv = s_qkv;   // conv1d weights [conv channel][4]: the channels of the qkv rows

    const GTensor* to = e.g.find("output.weight");
    if (!to) to = te;
    if (g > 1) {   // the head splits over the vocabulary, its rows gathered to every rank
        int r0 = 0, r1 = 0;
        qb_tp_rows((int)to->ne[1], rk, g, &r0, &r1);
        s_head.rows.push_back({r0, r1 - r0});
        head_row0 = r0;
    }
    if (upload_mat(e, to, e.output, tmp, tmp_bytes, s_head, head_row0)) return -1;
    if (!(e.out_norm = upload_f32(e, e.g.find("output_norm.weight")))) { set_err(-1, "output_norm"); return -1; }

    e.L.resize(d.n_layer);
    int nr = 0, na = 0;
    for (uint32_t il = 0; il < d.n_layer; ++il) {
        LayerW& l = e.L[il];
        l.rec = ((il + 1) % c.full_attn_interval) != 0;
        if (!(l.attn_norm = upload_f32(e, T("blk.%d.attn_norm.weight", il)))) return -1;
        if (!(l.post_norm = upload_f32(e, T("blk.%d.post_attention_norm.weight", il)))) return -1;
        if (upload_mat(e, T("blk.%d.ffn_gate.weight", il), l.ffn_gate, tmp, tmp_bytes, s_up) ||
            upload_mat(e, T("blk.%d.ffn_up.weight", il), l.ffn_up, tmp, tmp_bytes, s_up) ||
            upload_mat(e, T("blk.%d.ffn_down.weight", il), l.ffn_down, tmp, tmp_bytes, s_down) || build_gu(e, l))
            return -1;
        if (l.rec) {
            l.ridx = nr++;
            if (upload_mat(e, T("blk.%d.attn_qkv.weight", il), l.wqkv, tmp, tmp_bytes, s_qkv) ||
                upload_mat(e, T("blk.%d.attn_gate.weight", il), l.wgate, tmp, tmp_bytes, s_z) ||
                upload_mat(e, T("blk.%d.ssm_beta.weight", il), l.wbeta, tmp, tmp_bytes, s_ba) ||
                upload_mat(e, T("blk.%d.ssm_alpha.weight", il), l.walpha, tmp, tmp_bytes, s_ba) ||
                upload_mat(e, T("blk.%d.ssm_out.weight", il), l.ssm_out, tmp, tmp_bytes, s_out))
                return -1;
            if (!(l.conv_w = upload_f32(e, T("blk.%d.ssm_conv1d.weight", il), s_conv)) ||
                !(l.dt_bias = upload_f32(e, T("blk.%d.ssm_dt.bias", il), s_vec)) ||
                !(l.ssm_a = upload_f32(e, T("blk.%d.ssm_a", il), s_vec)) ||
                !(l.ssm_norm = upload_f32(e, T("blk.%d.ssm_norm.weight", il))))
                return -1;
        } else {
            l.aidx = na++;
            if (upload_mat(e, T("blk.%d.attn_q.weight", il), l.q, tmp, tmp_bytes, s_q) ||
                upload_mat(e, T("blk.%d.attn_k.weight", il), l.k, tmp, tmp_bytes, s_kv) ||
                upload_mat(e, T("blk.%d.attn_v.weight", il), l.v, tmp, tmp_bytes, s_kv) ||
                upload_mat(e, T("blk.%d.attn_output.weight", il), l.o, tmp, tmp_bytes, s_o))
                return -1;
            if (!(l.q_norm = upload_f32(e, T("blk.%d.attn_q_norm.weight", il))) ||
                !(l.k_norm = upload_f32(e, T("blk.%d.attn_k_norm.weight", il))))
                return -1;
        }
    }
    d.n_recr_layer = nr;
    d.n_attn_layer = na;
    {   // MTP block blk.<n_layer>
        const int im = (int)d.n_layer;
        LayerW& l = e.mtp;
        if (!(l.attn_norm = upload_f32(e, T("blk.%d.attn_norm.weight", im)))) return -1;
        if (!(l.post_norm = upload_f32(e, T("blk.%d.post_attention_norm.weight", im)))) return -1;
        if (upload_mat(e, T("blk.%d.attn_q.weight", im), l.q, tmp, tmp_bytes, s_q) ||
            upload_mat(e, T("blk.%d.attn_k.weight", im), l.k, tmp, tmp_bytes, s_kv) ||
            upload_mat(e, T("blk.%d.attn_v.weight", im), l.v, tmp, tmp_bytes, s_kv) ||
            upload_mat(e, T("blk.%d.attn_output.weight", im), l.o, tmp, tmp_bytes, s_o) ||
            upload_mat(e, T("blk.%d.ffn_gate.weight", im), l.ffn_gate, tmp, tmp_bytes, s_up) ||
            upload_mat(e, T("blk.%d.ffn_up.weight", im), l.ffn_up, tmp, tmp_bytes, s_up) ||
            upload_mat(e, T("blk.%d.ffn_down.weight", im), l.ffn_down, tmp, tmp_bytes, s_down) ||
            upload_mat(e, T("blk.%d.nextn.eh_proj.weight", im), e.eh_proj, tmp, tmp_bytes) || build_gu(e, l))
            return -1;
        if (!(l.q_norm = upload_f32(e, T("blk.%d.attn_q_norm.weight", im))) ||
            !(l.k_norm = upload_f32(e, T("blk.%d.attn_k_norm.weight", im))) ||
            !(e.enorm = upload_f32(e, T("blk.%d.nextn.enorm.weight", im))) ||
            !(e.hnorm = upload_f32(e, T("blk.%d.nextn.hnorm.weight", im))) ||
            !(e.shnorm = upload_f32(e, T("blk.%d.nextn.shared_head_norm.weight", im))))
            return -1;
        if (e.eh_proj.K != 2 * e.E || e.eh_proj.rows_all != e.E) { set_err(-1, "eh_proj shape"); return -1; }
    }

    // ---- states ----
    e.conv_layer = (size_t)(2 * e.nk_loc * dk + e.nv_loc * (int)d.head_v_dim) * 4;
    e.ssm_layer = (size_t)e.nv_loc * d.head_v_dim * d.head_k_dim;
    e.conv_slot_stride = e.conv_layer * nr;
    e.ssm_slot_stride = e.ssm_layer * nr;
    e.conv_slots = (float*)e.dalloc(std::max<size_t>(1, e.conv_slot_stride * kNSlot) * 4);
    e.ssm_slots = (float*)e.dalloc(std::max<size_t>(1, e.ssm_slot_stride * kNSlot) * 4);
    e.kv_layer = (size_t)n_ctx * e.nkv_loc * d.head_dim;
    e.kv_k = (float*)e.dalloc(std::max<size_t>(1, e.kv_layer * na) * 4);
    e.kv_v = (float*)e.dalloc(std::max<size_t>(1, e.kv_layer * na) * 4);
    e.mtp_k = (float*)e.dalloc(e.kv_layer * 4);
    e.mtp_v = (float*)e.dalloc(e.kv_layer * 4);
    if (!e.conv_slots || !e.ssm_slots || !e.kv_k || !e.kv_v || !e.mtp_k || !e.mtp_v) {
        set_err(-2, "state allocation failed");
        return -1;
    }
    CK(cudaMemset(e.conv_slots, 0, std::max<size_t>(1, e.conv_slot_stride * kNSlot) * 4));
    CK(cudaMemset(e.ssm_slots, 0, std::max<size_t>(1, e.ssm_slot_stride * kNSlot) * 4));
    CK(cudaMemset(e.kv_k, 0, std::max<size_t>(1, e.kv_layer * na) * 4));
    CK(cudaMemset(e.kv_v, 0, std::max<size_t>(1, e.kv_layer * na) * 4));
    CK(cudaMemset(e.mtp_k, 0, e.kv_layer * 4));
    CK(cudaMemset(e.mtp_v, 0, e.kv_layer * 4));

    // RoPE tables on the host with the reference's libm calls (src/model.c:186-201)
    {
        const int half = e.rope_half;
        std::vector<float> cs((size_t)n_ctx * half), sn((size_t)n_ctx * half);
        for (int p = 0; p < (int)n_ctx; ++p)
            for (int i = 0; i < half; ++i) {
                const float angle = (float)p * powf(c.rope_theta, -2.0f * (float)i / (float)c.rope_dim_count);
                cs[(size_t)p * half + i] = cosf(angle);
                sn[(size_t)p * half + i] = sinf(angle);
            }
        e.rope_cos = (float*)e.dalloc(cs.size() * 4);
        e.rope_sin = (float*)e.dalloc(sn.size() * 4);
        if (!e.rope_cos || !e.rope_sin) { set_err(-2, "rope alloc"); return -1; }
        CK(cudaMemcpyAsync(e.rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, e.st));
        CK(cudaMemcpyAsync(e.rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, e.st));
        CK(cudaStreamSynchronize(e.st));
    }

    // ---- activations: QB_WIDE rows (multi-sequence forwards), QB_MAX_TOK for the
    // tensor-parallel partial sums and the input preparation chunks ----
    const int T8 = QB_MAX_TOK, TW = QB_WIDE;
    e.ld_qkv = std::max<int>({(int)d.conv_dim, 2 * (int)d.n_head * (int)d.head_dim, e.F, 2 * e.E});
    auto A = [&](size_t n) { return (float*)e.dalloc(n * 4); };
    {   // every buffer a GEMV writes, plus the TP flags, in one arena (peers map it)
        const size_t sz[12] = {(size_t)TW * e.E,      (size_t)TW * e.ld_qkv,   (size_t)TW * d.d_inner,
                               (size_t)TW * 256,      (size_t)TW * 256,        (size_t)TW * 2 * d.n_head * d.head_dim,
                               (size_t)TW * 2 * d.n_kv_head * d.head_dim,      (size_t)TW * e.F,
                               (size_t)TW * e.F,      (size_t)TW * e.V,        (size_t)TW * e.E,
                               (size_t)TW * e.V};
        float** dst[12] = {&e.bx, &e.qkv, &e.z, &e.beta, &e.alpha, &e.qbuf, &e.kvbuf, &e.gate, &e.up, &e.logits,
                           &e.mtp_x, &e.mtp_logits};
        size_t off[12], total = 0;
        for (int i = 0; i < 12; ++i) {
            off[i] = total;
            total += (sz[i] * 4 + 255) / 256 * 256;
        }
        const size_t flags_off = total;   // TP barrier flags, then the argmax exchange words
        total += 256 + 2 * QB_TP_MAX * QB_MAX_TOK * 16;
        const size_t part_off = total;   // tensor parallelism: 2 slots of partial sums
        total += 2 * (size_t)T8 * e.E * 8;
        e.arena = (char*)e.dalloc(total);
        if (!e.arena) { set_err(-2, "activation arena alloc"); return -1; }
        e.arena_bytes = total;
        CK(cudaMemset(e.arena, 0, total));
        for (int i = 0; i < 12; ++i) *dst[i] = (float*)(e.arena + off[i]);
        e.tp.flags = (unsigned*)(e.arena + flags_off);
        e.ax.xk = (unsigned long long*)(e.arena + flags_off + 256);
        e.part = (uint2*)(e.arena + part_off);
        e.tp.part = e.part;
        e.tp.part_slot = (long long)T8 * e.E;
    }
    e.h_save = A((size_t)TW * e.E);
    e.qkvc = A((size_t)TW * e.ld_qkv);
    e.o = A((size_t)TW * d.d_inner);
    e.y = A((size_t)TW * d.d_inner);
    e.attn_o = A((size_t)TW * d.n_head * d.head_dim);
    e.act = A((size_t)TW * e.F);
    e.mtp_h = A((size_t)e.E);
    e.emb = A((size_t)TW * e.E);
    e.wam = (uint32_t*)e.dalloc(2 * (size_t)TW * 4);
    const int Kmax = std::max<int>({2 * e.E, e.F, (int)d.d_inner, (int)(d.n_head * d.head_dim)});
    // the GEMV input: QB_WIDE / QB_MAX_TOK chunks of QB_MAX_TOK rows (QbXBuf chunk strides)
    const int NC = TW / T8;
    e.xb.cs_frag = (long long)(qb_xfrag_bytes(Kmax) / sizeof(uint2));
    e.xb.cs_q = (long long)(qb_xq_bytes(Kmax) / sizeof(uint2));
    e.xb.xfrag = (uint2*)e.dalloc(NC * qb_xfrag_bytes(Kmax));
    e.xb.xscale = A((size_t)NC * T8 * (Kmax / 256));
    e.xb.xsum = A((size_t)NC * T8 * (Kmax / 32));
    e.xb.xq = (uint2*)e.dalloc(NC * qb_xq_bytes(Kmax));
    e.xb.xqscale = A((size_t)NC * T8 * (Kmax / 256));
    e.xb.xtc = (uint8_t*)e.dalloc(qb_xtc_bytes(Kmax));
    e.xb.xtc16 = (uint8_t*)e.dalloc(qb_xtc16_bytes(Kmax));   // wide inputs on qb_qmv_tcw
    e.xb.xtc32 = (uint8_t*)e.dalloc(qb_xtc32_bytes(Kmax));
    if (!e.xb.xtc16 || !e.xb.xtc32) { set_err(-2, "activation alloc"); return -1; }
    if (!e.xb.xtc) { set_err(-2, "activation alloc"); return -1; }
    if (e.fuse) {
        e.xb_alt.xfrag = (uint2*)e.dalloc(qb_xfrag_bytes(Kmax));
        e.xb_alt.xscale = A((size_t)T8 * (Kmax / 256));
        e.xb_alt.xsum = A((size_t)T8 * (Kmax / 32));
        e.xb_alt.xq = (uint2*)e.dalloc(qb_xq_bytes(Kmax));
        e.xb_alt.xqscale = A((size_t)T8 * (Kmax / 256));
        e.ss = A((size_t)T8 * (Kmax / 256));
        if (!e.xb_alt.xfrag || !e.xb_alt.xq || !e.ss) { set_err(-2, "activation alloc"); return -1; }
        CK(cudaMemset(e.xb_alt.xfrag, 0, qb_xfrag_bytes(Kmax)));
        CK(cudaMemset(e.xb_alt.xq, 0, qb_xq_bytes(Kmax)));
        CK(cudaMemset(e.xb_alt.xscale, 0, (size_t)T8 * (Kmax / 256) * 4));
        CK(cudaMemset(e.xb_alt.xqscale, 0, (size_t)T8 * (Kmax / 256) * 4));
        CK(cudaMemset(e.xb_alt.xsum, 0, (size_t)T8 * (Kmax / 32) * 4));
    }
    CK(cudaMemset(e.xb.xtc, 0, qb_xtc_bytes(Kmax)));
    CK(cudaMemset(e.xb.xtc16, 0, qb_xtc16_bytes(Kmax)));
    CK(cudaMemset(e.xb.xtc32, 0, qb_xtc32_bytes(Kmax)));
    {
        // chunk partials of up to kAttnGroups query groups (a 32-token prefill chunk)
        const size_t q_rows = (size_t)kAttnGroups * d.n_head * T8 * qb_attn_max_chunks((int)e.n_ctx);
        e.attn_po = A(q_rows * d.head_dim);
        e.attn_pml = (float2*)e.dalloc(q_rows * sizeof(float2));
        if (!e.attn_po || !e.attn_pml) { set_err(-2, "attention scratch alloc"); return -1; }
    }
    e.gates = (float2*)e.dalloc((size_t)TW * 256 * sizeof(float2));
    e.keys = (unsigned long long*)e.dalloc(2 * TW * sizeof(unsigned long long));
    e.ctrl = (QbCtrl*)e.dalloc(sizeof(QbCtrl));
    e.d_prompt = (uint32_t*)e.dalloc((size_t)e.n_ctx * 4);
    if (!e.bx || !e.logits || !e.xb.xfrag || !e.xb.xq || !e.ctrl || !e.emb || !e.keys || !e.d_prompt || !e.wam) {
        set_err(-2, "activation alloc");
        return -1;
    }
    CK(cudaMemset(e.xb.xfrag, 0, NC * qb_xfrag_bytes(Kmax)));
    CK(cudaMemset(e.xb.xscale, 0, (size_t)NC * T8 * (Kmax / 256) * 4));
    CK(cudaMemset(e.xb.xsum, 0, (size_t)NC * T8 * (Kmax / 32) * 4));
    CK(cudaMemset(e.xb.xq, 0, NC * qb_xq_bytes(Kmax)));
    CK(cudaMemset(e.xb.xqscale, 0, (size_t)NC * T8 * (Kmax / 256) * 4));
    CK(cudaMemset(e.wam, 0, 2 * (size_t)TW * 4));
    CK(cudaMemset(e.ctrl, 0, sizeof(QbCtrl)));
    CK(cudaMemset(e.mtp_h, 0, (size_t)e.E * 4));
    {   // GEMV scratch: arrival counters for the largest launch (head or fused FFN / mixer)
        const int max_pairs = (e.V + 31) / 32 + (2 * e.F + e.ld_qkv) / 32 + 64;
        CK(qb_qmv_work_alloc(e.work, max_pairs));
    }
    CK(cudaEventCreate(&e.ev0));
    CK(cudaEventCreate(&e.ev1));
    CK(cudaDeviceSynchronize());
    e.conv_base = e.conv_slots;
    e.ssm_base = e.ssm_slots;
    e.kv_k_base = e.kv_k;
    e.kv_v_base = e.kv_v;
    e.mtp_k_base = e.mtp_k;
    e.mtp_v_base = e.mtp_v;
    e.mtp_h_base = e.mtp_h;
    e.ctrl_base = e.ctrl;
    e.seq_pos.assign(1, 0u);
    return 0;
}

// ----------------------------- launch helpers ---------------------------------

// How a GEMV runs under tensor parallelism (tp_world > 1):
enum TpMode {
    TP_LOCAL = 0,     // this rank's output rows (heads / FFN columns) stay here: no exchange
    TP_PARTIAL = 1,   // this rank's input columns: partial sums, then qb_tp_reduce into the output
    TP_GATHER = 2,    // this rank's rows stored into every rank's output (the vocabulary head)
};

// y = W x for every matrix of mats (one input, e.xb).  With epi (one matrix)
// the launch also prepares the next input into e.xb_alt, which then becomes e.xb.
int gemv_group(Engine& e, const DevMat* const* mats, float* const* outs, const long long* ldos, int nm, int K,
               int N, int accumulate, const QbEpi* epi = nullptr, int tp_mode = TP_LOCAL) {
    if (epi && nm != 1) { set_err(-1, "fused epilogue on a multi-matrix GEMV"); return -1; }
    if (N > QB_MAX_TOK) {   // wide input (multi-sequence forward): one weight sweep per chunk of QB_MAX_TOK rows
        if (N > QB_WIDE || nm > QB_MAX_SEG * 4 || epi || e.xss || e.use_tc || e.tp_world > 1) {
            set_err(-1, "wide GEMV: at most %d rows, no fused epilogue, one GPU", QB_WIDE);
            return -1;
        }
        // IQ4_XS with tcgen05 tiles: all rows in one sweep on the tensor cores; the
        // other matrices in 8-row chunks (xp_needs prepared both input formats)
        const DevMat* rest[QB_MAX_SEG * 4];
        float* rest_out[QB_MAX_SEG * 4];
        long long rest_ld[QB_MAX_SEG * 4];
        int nr = 0;
        QbQSeg segs[QB_MAX_SEG];
        int ns = 0;
        auto flush = [&]() -> int {
            if (ns) CK(qb_qmv_tcw(segs, ns, K, N, e.xb, accumulate, 0, 1 << 30, e.work, e.st));
            ns = 0;
            return 0;
        };
        for (int i = 0; i < nm; ++i) {
            if (e.tcw && mats[i]->type == QB_IQ4_XS && mats[i]->w_tc) {
                if (mats[i]->rows == 0) continue;
                if (ns == QB_MAX_SEG && flush()) return -1;
                segs[ns].w = mats[i]->w_tc;
                segs[ns].out = outs[i] + mats[i]->row0;
                segs[ns].ldo = ldos[i];
                segs[ns].rows = mats[i]->rows;
                ++ns;
            } else {
                rest[nr] = mats[i];
                rest_out[nr] = outs[i];
                rest_ld[nr] = ldos[i];
                ++nr;
            }
        }
        if (flush()) return -1;
        e.xready = false;
        if (nr == 0) return 0;
        mats = rest;
        outs = rest_out;
        ldos = rest_ld;
        nm = nr;
        const QbXBuf xb0 = e.xb;
        for (int c = 0; c * QB_MAX_TOK < N; ++c) {
            float* oc[QB_MAX_SEG * 4];
            for (int i = 0; i < nm; ++i) oc[i] = outs[i] + (size_t)c * QB_MAX_TOK * ldos[i];
            e.xb = qb_xb_chunk(xb0, c, K / 256);
            const int r = gemv_group(e, mats, oc, ldos, nm, K, std::min(QB_MAX_TOK, N - c * QB_MAX_TOK), accumulate,
                                     nullptr, tp_mode);
            e.xb = xb0;
            if (r) return -1;
        }
        return 0;
    }
    const QbInNorm in_norm{e.xss, e.eps};
    // fuse matrices of the same type; different types run as separate launches
    int i = 0;
    while (i < nm) {
        QbQSeg segs[QB_MAX_SEG];
        int ns = 0;
        const int type = mats[i]->type;
        int nt = 0;   // matrices of this launch (with or without rows on this rank)
        while (i < nm && nt < QB_MAX_SEG && mats[i]->type == type) {
            if (mats[i]->rows > 0) {   // tensor parallelism: this rank's rows land at their global index
                segs[ns].w = mats[i]->w;
                segs[ns].out = outs[i] + mats[i]->row0;
                segs[ns].ldo = ldos[i];
                segs[ns].rows = mats[i]->rows;
                ++ns;
            }
            ++nt;
            ++i;
        }
        if (e.tp_world > 1 && tp_mode != TP_LOCAL) {
            if (!e.tp_ready || type == QB_F32) { set_err(-1, "tensor-parallel GEMV before qb_tp_connect"); return -1; }
            QbTp tp = e.tp;
            tp.gather = tp_mode == TP_GATHER;
            CK(qb_qmv_ex(type, segs, ns, K, N, e.xb, tp.gather ? accumulate : 0, nullptr, nullptr, &tp, e.work, e.st));
            continue;
        }
        if (ns == 0) continue;   // tensor parallelism: no rows of this launch on this rank
        if (type == QB_F32) {
            for (int s = 0; s < ns; ++s) CK(cudaErrorNotSupported);
        } else if (type == QB_IQ4_XS && N <= 4 && e.use_tc) {
            if (e.xss || epi) { set_err(-1, "fused epilogues need the mma.sync GEMV"); return -1; }
            for (int s = 0; s < ns; ++s) segs[s].w = mats[i - nt + s]->w_tc;
            CK(qb_qmv_tc(segs, ns, K, N, e.xb, accumulate, 0, 1 << 30, e.work, e.st));
        } else {
            CK(qb_qmv_ex(type, segs, ns, K, N, e.xb, accumulate, &in_norm, epi, nullptr, e.work, e.st));
        }
    }
    e.xready = epi != nullptr;
    if (epi) {
        std::swap(e.xb, e.xb_alt);
        e.xss = epi->kind == QB_EPI_NORM ? epi->ss : nullptr;
    }
    return 0;
}

// The sequences of the forward being recorded: e.ms_S sequences of B / e.ms_S rows,
// control blocks sizeof(QbCtrl) apart, states `state` floats apart.
QbSeqs seqs(const Engine& e, int B, long long state) {
    return QbSeqs{e.ms_S, B / e.ms_S, (long long)(sizeof(QbCtrl) / 4), state, 0};
}
// where the verify / MTP heads leave their argmax: the control block of a single
// sequence, the flat per-row arrays of a multi-sequence forward
uint32_t* am_verify(Engine& e) { return e.ms_S > 1 ? e.wam : e.ctrl->argmax; }
uint32_t* am_mtp(Engine& e) { return e.ms_S > 1 ? e.wam + QB_WIDE : e.ctrl->mtp_argmax; }

// a kernel other than a GEMV epilogue is about to write e.xb
void fresh_input(Engine& e) {
    e.xss = nullptr;
    e.xready = false;
}

// Residual GEMV x += W h (x [N][E]).  Under tensor parallelism W holds this
// rank's input columns: partial sums, then every rank adds all ranks' partials
// in rank order (the all-reduce, by NVLink loads of the peers' slots).
int residual_gemv(Engine& e, const DevMat* m, float* x, int K, int N, const QbEpi* epi) {
    const DevMat* m1[1] = {m};
    float* o1[1] = {x};
    const long long ld1[1] = {e.E};
    if (e.tp_world == 1) return gemv_group(e, m1, o1, ld1, 1, K, N, 1, epi);
    if (gemv_group(e, m1, o1, ld1, 1, K, N, 0, nullptr, TP_PARTIAL)) return -1;
    CK(qb_tp_reduce(x, e.E, e.E, N, e.tp, e.peer_part, e.work.err, e.st));
    return 0;
}

// the qb_xprep outputs that the matrices consuming an input of N tokens read
int xp_needs(const Engine& e, std::initializer_list<const DevMat*> ms, int N) {
    int w = 0;
    for (const DevMat* m : ms) {
        if (e.tcw && N > QB_MAX_TOK && m->type == QB_IQ4_XS && m->w_tc)
            w |= N <= QB_TC16_TOK ? QB_XP_TC16 : QB_XP_TC32;   // qb_qmv_tcw, one sweep for all rows
        else
            w |= qb_xprep_needs(m->type, N, e.use_tc ? 1 : 0);
    }
    return w;
}

int xprep1(Engine& e, const float* x, long long ldx, const float* norm_w, int len, int N, int what) {
    fresh_input(e);
    QbXIn in{x, ldx, norm_w, len};
    CK(qb_xprep(&in, 1, N, e.eps, e.xb, what, e.st));
    return 0;
}

// The RMSNorm the residual stream gets next and the fragments its readers
// need: the residual GEMV before it prepares that input in its epilogue.
struct NextIn {
    const float* norm_w = nullptr;
    int what = 0;
};

// RMSNorm(x) * norm_w as the next GEMV input, unless the last GEMV's epilogue made it
int norm_input(Engine& e, const float* x, const float* norm_w, int B, int what) {
    if (e.xready) {
        e.xready = false;
        return 0;
    }
    return xprep1(e, x, e.E, norm_w, e.E, B, what);
}

// the epilogue that prepares next from a residual GEMV's output, or none
const QbEpi* residual_epi(Engine& e, const NextIn& next, QbEpi& buf) {
    if (!e.fuse || !next.norm_w) return nullptr;
    buf = QbEpi{QB_EPI_NORM, next.norm_w, e.ss, nullptr, 0, e.xb_alt, next.what};
    return &buf;
}

// SwiGLU FFN on residual x (src/model.c:819-842)
int ffn_block(Engine& e, const LayerW& l, float* x, int B, const NextIn& next) {
    if (l.gu.w) {
        if (norm_input(e, x, l.post_norm, B, xp_needs(e, {&l.gu}, B))) return -1;
        // gate / up GEMV whose epilogue writes h = silu(gate) * up and its fragments
        const QbEpi sw{QB_EPI_SWIGLU, nullptr, nullptr, e.act, e.F, e.xb_alt, xp_needs(e, {&l.ffn_down}, B)};
        const DevMat* m2[1] = {&l.gu};
        float* o2[1] = {e.act};
        const long long ld2[1] = {e.F};
        if (gemv_group(e, m2, o2, ld2, 1, e.E, B, 0, &sw)) return -1;
    } else {
        if (norm_input(e, x, l.post_norm, B, xp_needs(e, {&l.ffn_gate, &l.ffn_up}, B))) return -1;
        const DevMat* m2[2] = {&l.ffn_gate, &l.ffn_up};
        float* o2[2] = {e.gate, e.up};
        const long long ld2[2] = {e.F, e.F};
        if (gemv_group(e, m2, o2, ld2, 2, e.E, B, 0)) return -1;
        fresh_input(e);
        CK(qb_silu_mul_xprep(e.gate, e.up, e.F, e.F_loc, B, e.act, e.xb, xp_needs(e, {&l.ffn_down}, B), e.st));
    }
    QbEpi eb;
    return residual_gemv(e, &l.ffn_down, x, e.F_loc, B, residual_epi(e, next, eb));
}

// the readers of a layer's normed input: DeltaNet in-projections or q / k / v
NextIn layer_in(const Engine& e, const LayerW& l, int B) {
    if (l.rec) return {l.attn_norm, xp_needs(e, {&l.wqkv, &l.wgate, &l.wbeta, &l.walpha}, B)};
    return {l.attn_norm, xp_needs(e, {&l.q, &l.k, &l.v}, B)};
}

// the FFN's input: post-attention norm, read by gate / up
NextIn ffn_in(const Engine& e, const LayerW& l, int B) {
    return {l.post_norm, l.gu.w ? xp_needs(e, {&l.gu}, B) : xp_needs(e, {&l.ffn_gate, &l.ffn_up}, B)};
}

// gated attention block on residual x, positions *pos .. *pos+B-1
int attn_block(Engine& e, const LayerW& l, float* x, int B, const uint32_t* pos, float* kc, float* vc,
               long long kv_seq, const NextIn& next) {
    // a long prefill chunk: its queries in attn_groups groups over the one cache
    const QbSeqs sq = e.attn_groups > 1 ? QbSeqs{e.attn_groups, B / e.attn_groups, 0, 0, B / e.attn_groups}
                                        : seqs(e, B, kv_seq);
    // this rank's q-heads and kv-heads (all of them on one GPU)
    const qwen_dims_t& d = e.d;
    const int qw = 2 * d.n_head * d.head_dim, kvw = d.n_kv_head * d.head_dim, kvw_loc = e.nkv_loc * d.head_dim;
    if (norm_input(e, x, l.attn_norm, B, xp_needs(e, {&l.q, &l.k, &l.v}, B))) return -1;
    const DevMat* m3[3] = {&l.q, &l.k, &l.v};
    float* o3[3] = {e.qbuf, e.kvbuf, e.kvbuf + kvw_loc};
    const long long ld3[3] = {qw, 2 * kvw, 2 * kvw};
    if (gemv_group(e, m3, o3, ld3, 3, e.E, B, 0)) return -1;
    CK(qb_attn_prep(e.qbuf, qw, e.kvbuf, 2 * kvw, l.q_norm, l.k_norm, e.nh_loc, e.nkv_loc, d.head_dim,
                    e.rope_half, e.rope_cos, e.rope_sin, pos, B, e.eps, kc, vc, e.st, &sq));
    fresh_input(e);
    CK(qb_attn_decode(e.qbuf, qw, kc, vc, e.nh_loc, e.nkv_loc, d.head_dim, pos, B, e.n_ctx, e.attn_o,
                      e.nh_loc * d.head_dim, e.attn_po, e.attn_pml, e.xb, xp_needs(e, {&l.o}, B), e.st, &sq));
    QbEpi eb;
    if (residual_gemv(e, &l.o, x, e.nh_loc * d.head_dim, B, residual_epi(e, ffn_in(e, l, B), eb))) return -1;
    return ffn_block(e, l, x, B, next);
}

int gdn_block(Engine& e, const LayerW& l, int B, int ckpt, const NextIn& next) {
    // this rank's k-heads, their v-heads and conv channels (all of them on one GPU)
    const qwen_dims_t& d = e.d;
    const int conv_loc = 2 * e.nk_loc * (int)d.head_k_dim + e.nv_loc * (int)d.head_v_dim;
    const int inner_loc = e.nv_loc * (int)d.head_v_dim;
    if (norm_input(e, e.bx, l.attn_norm, B, xp_needs(e, {&l.wqkv, &l.wgate, &l.wbeta, &l.walpha}, B))) return -1;
    const DevMat* m4[4] = {&l.wqkv, &l.wgate, &l.wbeta, &l.walpha};
    float* o4[4] = {e.qkv, e.z, e.beta, e.alpha};
    const long long ld4[4] = {e.ld_qkv, d.d_inner, 256, 256};
    if (gemv_group(e, m4, o4, ld4, 4, e.E, B, 0)) return -1;
    float* conv = e.conv_slots + (size_t)l.ridx * e.conv_layer;
    float* ssm = e.ssm_slots + (size_t)l.ridx * e.ssm_layer;
    const QbSeqs sq_conv = seqs(e, B, e.seq_conv), sq_ssm = seqs(e, B, e.seq_ssm);
    CK(qb_gdn_conv(e.qkv, e.ld_qkv, conv_loc, B, l.conv_w, conv, e.conv_slot_stride, &e.ctrl->cur_slot, ckpt,
                   e.qkvc, e.ld_qkv, e.beta, e.alpha, 256, l.dt_bias, l.ssm_a, e.nv_loc, e.gates, e.st, &sq_conv));
    CK(qb_gdn_recur(e.qkvc, e.ld_qkv, e.gates, e.nk_loc, e.nv_loc, d.head_k_dim, B, e.eps, ssm,
                    e.ssm_slot_stride, &e.ctrl->cur_slot, ckpt, e.o, d.d_inner, e.st, &sq_ssm));
    fresh_input(e);
    if (d.head_v_dim == 128 && e.nv_loc % 2 == 0) {
        CK(qb_gdn_out_xprep(e.o, e.z, d.d_inner, l.ssm_norm, e.nv_loc, d.head_v_dim, B, e.eps, e.y, e.xb,
                            xp_needs(e, {&l.ssm_out}, B), e.st));
    } else {
        CK(qb_gdn_out(e.o, e.z, d.d_inner, l.ssm_norm, e.nv_loc, d.head_v_dim, B, e.eps, e.y, e.st));
        if (xprep1(e, e.y, d.d_inner, nullptr, inner_loc, B, xp_needs(e, {&l.ssm_out}, B))) return -1;
    }
    QbEpi eb;
    if (residual_gemv(e, &l.ssm_out, e.bx, inner_loc, B, residual_epi(e, ffn_in(e, l, B), eb))) return -1;
    return ffn_block(e, l, e.bx, B, next);
}

// Control-block and copy kernels of the decode graphs.  Launched like every other
// kernel (qb_launch: programmatic dependent launch), so that they do not break the
// chain of early launches the way plain launches and memcpy nodes do.
__global__ void set_u32_kernel(uint32_t* p, uint32_t v) {
    pdl_wait();
    pdl_trigger();
    *p = v;
}
// cur_slot of the control blocks of all sequences (one block each)
__global__ void set_slot_kernel(QbCtrl* c, uint32_t v) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) c[blockIdx.x].cur_slot = v;
}
__global__ void copy_f32_kernel(float* __restrict__ dst, const float* __restrict__ src, int n) {
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = src[i];
}
cudaError_t copy_f32(float* dst, const float* src, int n, cudaStream_t st) {
    const int blocks = std::min((n + 255) / 256, 64);
    return qb_launch(copy_f32_kernel, dim3(blocks), dim3(256), 0, st, dst, src, n);
}

// Output head on the prepared input e.xb: logits -> out[b], argmax -> am[b]
// (the greedy pick of src/model.c:746-756 over the full row).  Under tensor
// parallelism every rank computes its vocabulary rows; with local_rows they stay
// on their rank and the ranks exchange their row maxima instead (the decode
// graphs, which only need the index), otherwise each rank stores its rows into
// every rank's logits.
int head(Engine& e, float* out, int B, unsigned long long* keys, uint32_t* am, bool local_rows) {
    const DevMat* m1[1] = {&e.output};
    float* o1[1] = {out};
    const long long ld1[1] = {e.V};
    const bool xchg = e.tp_world > 1 && local_rows;
    if (gemv_group(e, m1, o1, ld1, 1, e.E, B, 0, nullptr, xchg ? TP_LOCAL : TP_GATHER)) return -1;
    CK(qb_argmax_reset(keys, B, e.st));
    if (xchg) {
        CK(qb_argmax(out + e.output.row0, e.V, e.output.rows, B, keys, e.st, e.output.row0));
        CK(qb_tp_argmax(keys, B, am, e.ax, e.st));
    } else {
        CK(qb_argmax(out, e.V, e.V, B, keys, e.st));
        CK(qb_argmax_to_u32(keys, B, am, e.st));
    }
    return 0;
}

// model_forward_batch on the device: tokens ctrl->fwd_tok[0..B), positions
// ctrl->fwd_pos + b.  Logits -> e.logits[b] (this rank's vocabulary rows only
// with local_rows under tensor parallelism), argmax -> ctrl->argmax[b].
// Without with_head (prefill chunks before the last) the output head and the
// argmax are skipped: only the states, the KV cache and h_save advance.
int fwd_backbone(Engine& e, int B, int ckpt, bool local_rows = false, bool with_head = true) {
    const QbSeqs sq_tok = seqs(e, B, 0);
    CK(qb_embed(e.embd_type, e.tok_embd, e.E, e.ctrl->fwd_tok, B, e.bx, e.E, e.st, &sq_tok));
    fresh_input(e);
    for (size_t il = 0; il < e.L.size(); ++il) {
        const LayerW& l = e.L[il];
        const NextIn next = il + 1 < e.L.size() ? layer_in(e, e.L[il + 1], B)
                                                : NextIn{e.out_norm, xp_needs(e, {&e.output}, B)};
        if (l.rec) {
            if (gdn_block(e, l, B, ckpt, next)) return -1;
        } else {
            float* kc = e.kv_k + (size_t)l.aidx * e.kv_layer;
            float* vc = e.kv_v + (size_t)l.aidx * e.kv_layer;
            if (attn_block(e, l, e.bx, B, &e.ctrl->fwd_pos, kc, vc, e.seq_kv, next)) return -1;
        }
    }
    CK(copy_f32(e.h_save, e.bx, B * e.E, e.st));
    if (with_head) {
        if (norm_input(e, e.bx, e.out_norm, B, xp_needs(e, {&e.output}, B))) return -1;
        if (head(e, e.logits, B, e.keys, am_verify(e), local_rows)) return -1;
    }
    if (ckpt) CK(qb_launch(set_slot_kernel, dim3(e.ms_S), dim3(1), 0, e.st, e.ctrl,
                           (uint32_t)std::min(B / e.ms_S - 1, kNSlot - 1)));
    CK(cudaGetLastError());
    return 0;
}

// mtp_forward(_batch) on the device: tokens ctrl->mtp_tok[0..B), positions
// ctrl->mtp_pos + b, hidden input = hsrc rows (mtp_h for the single-token
// chain, h_save for the batch fill).  mtp_h <- output of the last token.
int fwd_mtp(Engine& e, int B, const float* hsrc, int want_logits, bool local_rows = false) {
    if (e.ms_S > 1 && B != e.ms_S) { set_err(-1, "multi-sequence MTP step: one row per sequence"); return -1; }
    const QbSeqs sq_tok = seqs(e, B, 0);
    CK(qb_embed(e.embd_type, e.tok_embd, e.E, e.ctrl->mtp_tok, B, e.emb, e.E, e.st, &sq_tok));
    QbXIn in[2] = {{e.emb, e.E, e.enorm, e.E}, {hsrc, e.E, e.hnorm, e.E}};
    fresh_input(e);
    CK(qb_xprep(in, 2, B, e.eps, e.xb, xp_needs(e, {&e.eh_proj}, B), e.st));
    const DevMat* m1[1] = {&e.eh_proj};
    float* o1[1] = {e.mtp_x};
    const long long ld1[1] = {e.E};
    if (gemv_group(e, m1, o1, ld1, 1, 2 * e.E, B, 0)) return -1;
    const NextIn next = want_logits ? NextIn{e.shnorm, xp_needs(e, {&e.output}, B)} : NextIn{};
    if (attn_block(e, e.mtp, e.mtp_x, B, &e.ctrl->mtp_pos, e.mtp_k, e.mtp_v, e.seq_mtpkv, next)) return -1;
    if (e.ms_S > 1)   // every sequence's row: each sequence's MTP hidden
        CK(copy_f32(e.mtp_h, e.mtp_x, B * e.E, e.st));
    else
        CK(copy_f32(e.mtp_h, e.mtp_x + (size_t)(B - 1) * e.E, e.E, e.st));
    if (want_logits) {
        if (norm_input(e, e.mtp_x, e.shnorm, B, xp_needs(e, {&e.output}, B))) return -1;
        if (head(e, e.mtp_logits, B, e.keys + QB_WIDE, am_mtp(e), local_rows)) return -1;
    }
    return 0;
}

// ------------------------- speculative cycle kernels ----------------------------

// The cycle kernels run one block per sequence (blockIdx.x; one block for a single
// sequence): control block c + blockIdx.x.
//
// cycle start: cand[0] = next_cand0; first draft input = (cand[0], P+1)
__global__ void spec_start_kernel(QbCtrl* c) {
    pdl_wait();
    pdl_trigger();
    c += blockIdx.x;
    c->cand[0] = c->next_cand0;
    c->mtp_tok[0] = c->cand[0];
    c->mtp_pos = c->P + 1;
}
// after draft s: cand[s] = the draft's argmax (am[sequence]); next draft input = (cand[s], P+s+1)
__global__ void spec_draft_kernel(QbCtrl* c, int s, const uint32_t* am) {
    pdl_wait();
    pdl_trigger();
    const uint32_t a = am[blockIdx.x];
    c += blockIdx.x;
    c->cand[s] = a;
    c->mtp_tok[0] = c->cand[s];
    c->mtp_pos = c->P + s + 1;
}
__global__ void spec_verify_setup_kernel(QbCtrl* c, int k) {
    pdl_wait();
    pdl_trigger();
    c += blockIdx.x;
    for (int i = 0; i <= k; ++i) c->fwd_tok[i] = c->cand[i];
    c->fwd_pos = c->P + 1;
}
// acceptance (src/main.c:191-223): j = first i < k with argmax(logits_b[i])
// != cand[i+1], or the forced length; emit cand[0..j]; live slot = j; MTP
// anchor on (cand[j], h_save[j]) at P+j+1; next cand0 = argmax(logits_b[j]).
// Sequence q reads the verify argmax am[q (k+1) + i] and h_save rows q (k+1) + i,
// writes its tokens at out_tok + q * out_stride, its accept lengths at out_j + q *
// j_stride and its MTP hidden row mtp_h + q E.
__global__ void spec_accept_kernel(QbCtrl* c, int k, const uint32_t* forced, uint32_t* out_tok,
                                   uint32_t* out_j, const float* h_save, float* mtp_h, int E, const uint32_t* am,
                                   long long out_stride, long long j_stride) {
    pdl_wait();
    pdl_trigger();
    const int q = blockIdx.x;
    c += q;
    am += (size_t)q * (k + 1);
    out_tok += (size_t)q * out_stride;
    out_j += (size_t)q * j_stride;
    h_save += (size_t)q * (k + 1) * E;
    mtp_h += (size_t)q * E;
    __shared__ uint32_t sj;
    if (threadIdx.x == 0) {
        uint32_t j = (uint32_t)k;
        for (int i = 0; i < k; ++i)
            if (am[i] != c->cand[i + 1]) { j = (uint32_t)i; break; }
        if (c->n_forced) {
            j = forced[c->cycle % c->n_forced];
            if (j > (uint32_t)k) j = (uint32_t)k;
        }
        for (uint32_t i = 0; i <= j; ++i)
            if (c->n_out + i < c->cap_out) out_tok[c->n_out + i] = c->cand[i];
        if (c->cycle < c->cap_j) out_j[c->cycle] = j;
        c->n_out += j + 1;
        c->cycle += 1;
        c->j = j;
        c->cur_slot = j;                 // rollback = select the slot after token j
        const uint32_t P_new = c->P + j + 1;
        c->mtp_tok[0] = c->cand[j];
        c->mtp_pos = P_new;              // anchor position P + j + 1
        c->next_cand0 = am[j];
        c->P = P_new;
        sj = j;
    }
    __syncthreads();
    const float* src = h_save + (size_t)sj * E;
    for (int i = threadIdx.x; i < E; i += blockDim.x) mtp_h[i] = src[i];
}

// greedy decode step: next token = argmax of the previous forward
__global__ void greedy_step_kernel(QbCtrl* c, uint32_t* out_tok) {
    pdl_wait();
    pdl_trigger();
    const uint32_t t = c->argmax[0];
    if (c->greedy_n < c->cap_out) out_tok[c->greedy_n] = t;
    c->greedy_n += 1;
    c->fwd_tok[0] = t;
    c->fwd_pos += 1;
}

int record_cycle(Engine& e, int k) {
    const int S = e.ms_S;
    CK(qb_launch(spec_start_kernel, dim3(S), dim3(1), 0, e.st, e.ctrl));
    for (int s = 1; s <= k; ++s) {
        if (fwd_mtp(e, S, e.mtp_h, 1, true)) return -1;
        CK(qb_launch(spec_draft_kernel, dim3(S), dim3(1), 0, e.st, e.ctrl, s, (const uint32_t*)am_mtp(e)));
    }
    CK(qb_launch(spec_verify_setup_kernel, dim3(S), dim3(1), 0, e.st, e.ctrl, k));
    if (fwd_backbone(e, S * (k + 1), 1, true)) return -1;
    CK(qb_launch(spec_accept_kernel, dim3(S), dim3(256), 0, e.st, e.ctrl, k, (const uint32_t*)e.d_forced, e.d_out_tok,
                 e.d_out_j, (const float*)e.h_save, e.mtp_h, e.E, (const uint32_t*)am_verify(e),
                 (long long)e.cap_out, (long long)e.cap_j));
    if (fwd_mtp(e, S, e.mtp_h, 0)) return -1;
    CK(cudaGetLastError());
    return 0;
}

// prefill chunk start (src/main.c:137-146): the next B prompt tokens from the
// staged prompt at fwd_pos feed the backbone and, at the same positions, the MTP fill
__global__ void prefill_chunk_kernel(QbCtrl* c, const uint32_t* prompt, int B) {
    pdl_wait();
    pdl_trigger();
    const uint32_t p = c->fwd_pos;
    for (int i = 0; i < B; ++i) {
        c->fwd_tok[i] = prompt[p + i];
        c->mtp_tok[i] = prompt[p + i];
    }
    c->mtp_pos = p;
}
__global__ void prefill_advance_kernel(QbCtrl* c, int B) {
    pdl_wait();
    pdl_trigger();
    c->fwd_pos += (uint32_t)B;
}

// one full prefill chunk before the last: states, KV cache and h_save advance,
// no output head; with spec the MTP KV cache fills from h_save (src/model.c:1069-1103)
// arg: bit 0 spec, bit 1 a wide chunk (kPrefillW tokens: attention in kAttnGroups query
// groups, GEMVs of all rows at once)
int record_prefill(Engine& e, int arg) {
    const int spec = arg & 1, B = (arg & 2) ? kPrefillW : PREFILL_MAX_B;
    CK(qb_launch(prefill_chunk_kernel, dim3(1), dim3(1), 0, e.st, e.ctrl, (const uint32_t*)e.d_prompt, B));
    e.attn_groups = B / QB_MAX_TOK;
    int r = fwd_backbone(e, B, 0, false, false);
    if (!r && spec) r = fwd_mtp(e, B, e.h_save, 0);
    e.attn_groups = 1;
    if (r) return -1;
    CK(qb_launch(prefill_advance_kernel, dim3(1), dim3(1), 0, e.st, e.ctrl, B));
    CK(cudaGetLastError());
    return 0;
}

size_t g_last_graph_kernels = 0;

int capture(Engine& e, cudaGraphExec_t* out, int (*rec)(Engine&, int), int arg) {
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(e.st, cudaStreamCaptureModeThreadLocal));
    const int r = rec(e, arg);
    cudaError_t ce = cudaStreamEndCapture(e.st, &graph);
    if (r || ce != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        if (!r) CK(ce);
        return -1;
    }
    size_t n_nodes = 0, n_kern = 0;
    if (cudaGraphGetNodes(graph, nullptr, &n_nodes) == cudaSuccess && n_nodes) {
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        cudaGraphGetNodes(graph, nodes.data(), &n_nodes);
        for (auto nd : nodes) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++n_kern;
        }
    }
    g_last_graph_kernels = n_kern;
    cudaError_t ie = cudaGraphInstantiate(out, graph, 0);
    cudaGraphDestroy(graph);
    CK(ie);
    return 0;
}

// sampling decode step: the token just sampled goes out and feeds the next forward
__global__ void sample_step_kernel(QbCtrl* c, const QbSampDev* sd, uint32_t* out_tok, int advance) {
    pdl_wait();
    pdl_trigger();
    const uint32_t t = sd->token;
    if (c->greedy_n < c->cap_out) out_tok[c->greedy_n] = t;
    c->greedy_n += 1;
    c->fwd_tok[0] = t;
    if (advance) c->fwd_pos += 1;
}

// one step of src/main.c:241-242: forward of the previous token, then sample
int record_sample(Engine& e, int) {
    if (fwd_backbone(e, 1, 0, false)) return -1;   // every rank holds the whole logit row
    CK(qb_sample(e.logits, e.V, e.samp, e.samp_cand, e.samp_keys, e.samp_am, e.st));
    CK(qb_launch(sample_step_kernel, dim3(1), dim3(1), 0, e.st, e.ctrl, (const QbSampDev*)e.samp, e.d_out_tok, 1));
    CK(cudaGetLastError());
    return 0;
}

int record_greedy(Engine& e, int) {
    if (fwd_backbone(e, 1, 0, true)) return -1;
    CK(qb_launch(greedy_step_kernel, dim3(1), dim3(1), 0, e.st, e.ctrl, e.d_out_tok));
    CK(cudaGetLastError());
    return 0;
}

// Decode graphs under tensor parallelism leave in each row of e.logits only this
// rank's vocabulary rows: fetch the others of row `row` from the peers' copies.
// Every rank calls this at the same point.  The barrier before the loads orders
// them after every peer's last head GEMV; the one after keeps each peer's
// logits unchanged until all ranks have read them.
int tp_fill_logits_row(Engine& e, int row) {
    if (e.tp_world < 2) return 0;
    QbTp bar = e.tp;
    bar.gather = 1;
    CK(qb_qmv_ex(e.output.type, nullptr, 0, e.E, 1, e.xb, 0, nullptr, nullptr, &bar, e.work, e.st));
    float* dst = e.logits + (size_t)row * e.V;
    const float* src[QB_TP_MAX] = {};
    int r0[QB_TP_MAX] = {}, r1[QB_TP_MAX] = {};
    for (int r = 0; r < e.tp_world; ++r) {
        if (r != e.tp_rank) src[r] = (const float*)((char*)e.peer_arena[r] + ((char*)dst - e.arena));
        qb_tp_rows(e.V, r, e.tp_world, &r0[r], &r1[r]);
    }
    CK(qb_tp_pull_rows(dst, src, r0, r1, e.tp_world, e.tp_rank, e.st));
    CK(qb_qmv_ex(e.output.type, nullptr, 0, e.E, 1, e.xb, 0, nullptr, nullptr, &bar, e.work, e.st));
    return 0;
}

// The tcgen05 tile copy of an IQ4_XS matrix (qb_repack_tc of its GGUF rows), made on first use.
int ensure_w_tc(Engine& e, DevMat& m) {
    if (m.w_tc || m.type != QB_IQ4_XS || m.rows == 0) return 0;
    if (!m.src || m.rows != m.rows_all) { set_err(-1, "tcgen05 tiles need the whole matrix"); return -1; }
    const size_t src = gguf_row_bytes(m.src->type, m.src->ne[0]) * m.src->ne[1];
    void* tmp = nullptr;
    CK(cudaMalloc(&tmp, src));
    m.w_tc = e.dalloc(qb_repacked_bytes_tc(m.rows, m.K));
    // stream-ordered copy: a pageable cudaMemcpy may return before its DMA lands, and the
    // model's stream does not wait for the legacy stream
    cudaError_t ce = m.w_tc ? cudaMemcpyAsync(tmp, m.src->data, src, cudaMemcpyHostToDevice, e.st)
                            : cudaErrorMemoryAllocation;
    if (ce == cudaSuccess) ce = qb_repack_tc(tmp, m.rows, m.K, m.w_tc, e.st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e.st);
    cudaFree(tmp);
    CK(ce);
    return 0;
}

// tcgen05 tile copies of every IQ4_XS matrix: GEMV inputs of more than QB_MAX_TOK rows
// (prefill chunks, multi-sequence verifies) then run IQ4_XS on qb_qmv_tcw
int enable_tcw(Engine& e) {
    if (e.tcw) return 0;
    if (e.tp_world > 1 || e.fuse || e.use_tc) { set_err(-1, "wide tcgen05 GEMM: one GPU, default GEMV paths"); return -1; }
    auto each = [&](LayerW& l) {
        DevMat* ms[] = {&l.ffn_gate, &l.ffn_up, &l.ffn_down, &l.wqkv, &l.wgate, &l.wbeta, &l.walpha, &l.ssm_out,
                        &l.q, &l.k, &l.v, &l.o};
        for (DevMat* d : ms)
            if (d->w && ensure_w_tc(e, *d)) return -1;
        return 0;
    };
    for (LayerW& l : e.L)
        if (each(l)) return -1;
    if (each(e.mtp)) return -1;
    e.tcw = true;
    // graphs recorded before route wide inputs through the 8-row chunks
    cudaGraphExec_t* gs[] = {&e.g_mcycle, &e.g_prefill_w[0], &e.g_prefill_w[1]};
    for (cudaGraphExec_t* g : gs)
        if (*g) {
            cudaGraphExecDestroy(*g);
            *g = nullptr;
        }
    e.g_mcycle_k = -1;
    return 0;
}

int ensure_out_buffers(Engine& e, uint32_t n_out, uint32_t n_j, uint32_t n_forced) {
    if (n_out > e.cap_out || n_j > e.cap_j || n_forced > e.cap_forced) {
        // buffers captured in graphs: re-capture after reallocation
        if (e.g_cycle) { cudaGraphExecDestroy(e.g_cycle); e.g_cycle = nullptr; }
        if (e.g_mcycle) { cudaGraphExecDestroy(e.g_mcycle); e.g_mcycle = nullptr; }
        if (e.g_greedy) { cudaGraphExecDestroy(e.g_greedy); e.g_greedy = nullptr; }
        if (e.g_sample) { cudaGraphExecDestroy(e.g_sample); e.g_sample = nullptr; }
        const uint32_t co = std::max(n_out, std::max(e.cap_out, 4096u));
        const uint32_t cj = std::max(n_j, std::max(e.cap_j, 4096u));
        const uint32_t cf = std::max(n_forced, std::max(e.cap_forced, 1024u));
        uint32_t *a = nullptr, *b = nullptr, *f = nullptr;
        // per sequence: cap_out tokens and cap_j accept lengths
        CK(cudaMalloc(&a, (size_t)co * e.n_seq * 4));
        CK(cudaMalloc(&b, (size_t)cj * e.n_seq * 4));
        CK(cudaMalloc(&f, (size_t)cf * 4));
        if (e.d_out_tok) cudaFree(e.d_out_tok);
        if (e.d_out_j) cudaFree(e.d_out_j);
        if (e.d_forced) cudaFree(e.d_forced);
        e.d_out_tok = a;
        e.d_out_j = b;
        e.d_forced = f;
        e.cap_out = co;
        e.cap_j = cj;
        e.cap_forced = cf;
    }
    return 0;
}

Engine* E_(qwen_model_t* m) { return m ? (Engine*)m->eng : nullptr; }

// Wait for the stream; a kernel whose bounded wait gave up (a ring copy, a
// tensor-parallel peer) left a code in work.err, reported here as an error.
int dev_sync(Engine& e) {
    CK(cudaStreamSynchronize(e.st));
    unsigned code = 0;
    CK(cudaMemcpy(&code, e.work.err, sizeof code, cudaMemcpyDeviceToHost));
    if (code) {
        cudaMemset(e.work.err, 0, sizeof code);
        set_err(-3, "a device-side wait gave up (code %u: 2 weight copy, 4 tensor-parallel peer)", code);
        return -1;
    }
    return 0;
}

// Graphs record the state pointers of the sequence they were captured for.
void drop_graphs(Engine& e) {
    cudaGraphExec_t* gs[] = {&e.g_cycle,      &e.g_mcycle,      &e.g_greedy,       &e.g_sample,
                             &e.g_prefill[0], &e.g_prefill[1], &e.g_prefill_w[0], &e.g_prefill_w[1]};
    for (cudaGraphExec_t* g : gs)
        if (*g) {
            cudaGraphExecDestroy(*g);
            *g = nullptr;
        }
    e.g_cycle_k = e.g_mcycle_k = -1;
}

// Sequence s's recurrent slots, KV caches, control block and MTP hidden row become
// the ones the single-sequence paths use.
void select_seq(Engine& e, int s) {
    if (s == e.cur_seq) return;
    drop_graphs(e);
    e.conv_slots = e.conv_base + (size_t)s * e.seq_conv;
    e.ssm_slots = e.ssm_base + (size_t)s * e.seq_ssm;
    e.kv_k = e.kv_k_base + (size_t)s * e.seq_kv;
    e.kv_v = e.kv_v_base + (size_t)s * e.seq_kv;
    e.mtp_k = e.mtp_k_base + (size_t)s * e.seq_mtpkv;
    e.mtp_v = e.mtp_v_base + (size_t)s * e.seq_mtpkv;
    e.mtp_h = e.mtp_h_base + (size_t)s * e.E;
    e.ctrl = e.ctrl_base + s;
    e.cur_seq = s;
}

int sync_host_mirrors_after_batch(qwen_model_t* m, Engine& e, int B) {
    CK(cudaMemcpyAsync(m->logits_b, e.logits, (size_t)B * e.V * 4, cudaMemcpyDeviceToHost, e.st));
    CK(cudaMemcpyAsync(m->h_save, e.h_save, (size_t)B * e.E * 4, cudaMemcpyDeviceToHost, e.st));
    CK(cudaStreamSynchronize(e.st));
    return 0;
}

}  // namespace

// ================================ C API: model ===================================

struct pool { int n; };

extern "C" pool_t* pool_create(int n_threads, int) {
    pool_t* p = (pool_t*)calloc(1, sizeof(pool_t));
    if (p) p->n = n_threads < 1 ? 1 : n_threads;
    return p;
}
extern "C" void pool_destroy(pool_t* p) { free(p); }
extern "C" void pool_run(pool_t*, pool_fn_t fn, void* arg) { fn(arg, 0, 1); }

extern "C" int model_init(qwen_model_t* m, const char* path, uint32_t n_ctx) {
    return qb_model_init_tp(m, path, n_ctx, 0, 1);
}

extern "C" int qb_model_init_tp(qwen_model_t* m, const char* path, uint32_t n_ctx, int rank, int world) {
    if (!m || !path || world < 1 || world > QB_TP_MAX || rank < 0 || rank >= world) return -1;
    memset(m, 0, sizeof *m);
    Engine* e = new Engine();
    e->tp_rank = rank;
    e->tp_world = world;
    e->tp.rank = rank;
    e->tp.world = world;
    if (engine_init(*e, path, n_ctx)) {
        delete e;
        return -1;
    }
    m->eng = e;
    m->cfg = e->cfg;
    m->dims = e->d;
    m->n_ctx = n_ctx;
    m->pos = 0;
    const size_t VB = (size_t)PREFILL_MAX_B * e->V, EB = (size_t)PREFILL_MAX_B * e->E;
    if (cudaMallocHost(&m->logits_b, VB * 4) != cudaSuccess || cudaMallocHost(&m->logits, (size_t)e->V * 4) != cudaSuccess ||
        cudaMallocHost(&m->h_save, EB * 4) != cudaSuccess || cudaMallocHost(&m->mtp_h, (size_t)e->E * 4) != cudaSuccess ||
        cudaMallocHost(&m->x, (size_t)e->E * 4) != cudaSuccess) {
        set_err(-2, "pinned host mirrors");
        model_free(m);
        return -1;
    }
    memset(m->mtp_h, 0, (size_t)e->E * 4);
    m->layers = (qwen_layer_t*)calloc(e->L.size() ? e->L.size() : 1, sizeof(qwen_layer_t));
    if (!m->layers) {
        set_err(-2, "layer table");
        model_free(m);
        return -1;
    }
    for (size_t il = 0; il < e->L.size(); ++il) {
        m->layers[il].index = (uint32_t)il;
        m->layers[il].is_recurrent = e->L[il].rec;
    }
    return 0;
}

extern "C" int64_t qb_tp_handle(qwen_model_t* m, void* out, int64_t cap) {
    Engine* e = E_(m);
    if (!e || !out || cap < (int64_t)sizeof(cudaIpcMemHandle_t)) return -1;
    cudaSetDevice(e->dev);
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, e->arena) != cudaSuccess) { set_err(-2, "cudaIpcGetMemHandle"); return -1; }
    memcpy(out, &h, sizeof h);
    return (int64_t)sizeof h;
}

extern "C" int qb_tp_connect(qwen_model_t* m, const void* handles, int64_t stride) {
    Engine* e = E_(m);
    if (!e || !handles || stride < (int64_t)sizeof(cudaIpcMemHandle_t) || e->tp_world < 2 || e->tp_ready) return -1;
    cudaSetDevice(e->dev);
    int q = 0;
    for (int r = 0; r < e->tp_world; ++r) {
        if (r == e->tp_rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const char*)handles + (size_t)r * stride, sizeof h);
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            set_err(-2, "cudaIpcOpenMemHandle (rank %d)", r);
            return -1;
        }
        e->peer_arena[r] = p;
        e->tp.delta[q++] = (long long)((char*)p - e->arena);
        e->peer_part[r] = (const void*)((char*)p + ((char*)e->part - e->arena));
    }
    e->peer_part[e->tp_rank] = e->part;
    e->ax.rank = e->tp_rank;
    e->ax.world = e->tp_world;
    for (int r = 0; r < e->tp_world; ++r)
        e->ax.delta[r] = r == e->tp_rank ? 0 : (long long)((char*)e->peer_arena[r] - e->arena);
    e->ax.err = e->work.err;
    e->tp.done = (unsigned*)e->dalloc(256);
    if (!e->tp.done) { set_err(-2, "tp counters"); return -1; }
    e->tp.seq = e->tp.done + 32;
    e->ax.xseq = e->tp.done + 48;
    if (cudaMemset(e->tp.done, 0, 256) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        set_err(-2, "tp counters");
        return -1;
    }
    e->tp_ready = true;
    return 0;
}

extern "C" void model_free(qwen_model_t* m) {
    if (!m) return;
    delete E_(m);
    if (m->logits_b) cudaFreeHost(m->logits_b);
    if (m->logits) cudaFreeHost(m->logits);
    if (m->h_save) cudaFreeHost(m->h_save);
    if (m->mtp_h) cudaFreeHost(m->mtp_h);
    if (m->x) cudaFreeHost(m->x);
    free(m->layers);
    memset(m, 0, sizeof *m);
}

static int do_forward_batch(qwen_model_t* m, const uint32_t* tokens, uint32_t pos, uint32_t B, int ckpt) {
    Engine* e = E_(m);
    if (!e || B < 1 || B > QB_MAX_TOK || pos + B > (uint32_t)e->n_ctx) {
        set_err(-1, "model_forward_batch: bad arguments (B=%u pos=%u)", B, pos);
        return -1;
    }
    CK(cudaSetDevice(e->dev));
    CK(cudaMemcpyAsync(e->ctrl->fwd_tok, tokens, B * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(&e->ctrl->fwd_pos, &pos, 4, cudaMemcpyHostToDevice, e->st));
    if (fwd_backbone(*e, (int)B, ckpt)) return -1;
    if (sync_host_mirrors_after_batch(m, *e, (int)B)) return -1;
    m->pos = pos + B;
    return 0;
}

// one layer of one token on m->x (attention_layer / gdn_layer)
static void one_layer(qwen_model_t* m, const qwen_layer_t* L, uint32_t pos, bool want_rec, const char* who) {
    Engine* e = E_(m);
    if (!e || !L || L->index >= e->L.size() || e->L[L->index].rec != want_rec) {
        set_err(-1, "%s: bad model or layer", who);
        return;
    }
    if (cudaSetDevice(e->dev) != cudaSuccess) { set_err(-2, "%s: device", who); return; }
    const LayerW& l = e->L[L->index];
    auto fail = [&]() { set_err(-2, "%s: CUDA failure", who); };
    if (cudaMemcpyAsync(e->bx, m->x, (size_t)e->E * 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess ||
        cudaMemcpyAsync(&e->ctrl->fwd_pos, &pos, 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess)
        return fail();
    fresh_input(*e);
    e->xready = false;
    const NextIn next = layer_in(*e, l, 1);
    int r;
    if (l.rec) {
        r = gdn_block(*e, l, 1, 0, next);
    } else {
        float* kc = e->kv_k + (size_t)l.aidx * e->kv_layer;
        float* vc = e->kv_v + (size_t)l.aidx * e->kv_layer;
        r = attn_block(*e, l, e->bx, 1, &e->ctrl->fwd_pos, kc, vc, 0, next);
    }
    fresh_input(*e);
    e->xready = false;
    if (r) return;
    if (cudaMemcpyAsync(m->x, e->bx, (size_t)e->E * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) return fail();
    dev_sync(*e);
}

extern "C" void attention_layer(qwen_model_t* m, qwen_layer_t* L, pool_t*, uint32_t pos) {
    one_layer(m, L, pos, false, "attention_layer");
}

extern "C" void gdn_layer(qwen_model_t* m, qwen_layer_t* L, pool_t*) {
    one_layer(m, L, 0, true, "gdn_layer");
}

extern "C" void model_forward(qwen_model_t* m, pool_t*, uint32_t token, uint32_t pos) {
    if (do_forward_batch(m, &token, pos, 1, 0)) return;
    Engine* e = E_(m);
    memcpy(m->logits, m->logits_b, (size_t)e->V * 4);
    memcpy(m->x, m->h_save, (size_t)e->E * 4);
}

extern "C" void model_forward_batch(qwen_model_t* m, pool_t*, const uint32_t* tokens, uint32_t pos, uint32_t B,
                                    int ckpt) {
    do_forward_batch(m, tokens, pos, B, ckpt);
}

extern "C" int model_snapshot_states(qwen_model_t*) { return 0; }
extern "C" void model_rollback_states(qwen_model_t*) {}

extern "C" void model_rollback_to(qwen_model_t* m, uint32_t b) {
    Engine* e = E_(m);
    if (!e || b >= (uint32_t)kNSlot) { set_err(-1, "model_rollback_to: bad slot %u", b); return; }
    cudaSetDevice(e->dev);
    set_u32_kernel<<<1, 1, 0, e->st>>>(&e->ctrl->cur_slot, b);
    cudaError_t ce = cudaStreamSynchronize(e->st);
    if (ce != cudaSuccess) set_err((int)ce, "model_rollback_to: %s", cudaGetErrorString(ce));
}

static int do_mtp(qwen_model_t* m, const uint32_t* tokens, uint32_t pos, uint32_t B, int want_logits, bool batch) {
    Engine* e = E_(m);
    if (!e || B < 1 || B > QB_MAX_TOK || pos + B > (uint32_t)e->n_ctx) {
        set_err(-1, "mtp_forward: bad arguments");
        return -1;
    }
    CK(cudaSetDevice(e->dev));
    CK(cudaMemcpyAsync(e->ctrl->mtp_tok, tokens, B * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(&e->ctrl->mtp_pos, &pos, 4, cudaMemcpyHostToDevice, e->st));
    const float* hsrc = e->mtp_h;
    if (batch) {
        // h_save rows as the hidden input (src/model.c:1077-1084): the caller's host
        // mirror is the source of truth, as for every other mirror
        CK(cudaMemcpyAsync(e->h_save, m->h_save, (size_t)B * e->E * 4, cudaMemcpyHostToDevice, e->st));
        hsrc = e->h_save;
    } else {
        CK(cudaMemcpyAsync(e->mtp_h, m->mtp_h, (size_t)e->E * 4, cudaMemcpyHostToDevice, e->st));
    }
    if (fwd_mtp(*e, (int)B, hsrc, want_logits)) return -1;
    CK(cudaMemcpyAsync(m->mtp_h, e->mtp_h, (size_t)e->E * 4, cudaMemcpyDeviceToHost, e->st));
    if (want_logits) {
        if (batch)
            CK(cudaMemcpyAsync(m->logits_b, e->mtp_logits, (size_t)B * e->V * 4, cudaMemcpyDeviceToHost, e->st));
        else
            CK(cudaMemcpyAsync(m->logits, e->mtp_logits, (size_t)e->V * 4, cudaMemcpyDeviceToHost, e->st));
    }
    if (dev_sync(*e)) return -1;
    return 0;
}

extern "C" int mtp_forward(qwen_model_t* m, pool_t*, uint32_t token, uint32_t pos, int want_logits) {
    do_mtp(m, &token, pos, 1, want_logits, false);
    return 0;   // the reference always returns 0 (src/model.c:1062)
}

extern "C" int mtp_forward_batch(qwen_model_t* m, pool_t*, const uint32_t* tokens, uint32_t pos, uint32_t B,
                                 int want_logits) {
    do_mtp(m, tokens, pos, B, want_logits, true);
    return 0;
}

extern "C" uint32_t qb_last_argmax(qwen_model_t* m, uint32_t b) {
    Engine* e = E_(m);
    if (!e || b >= QB_MAX_TOK) return 0;
    uint32_t v = 0;
    cudaSetDevice(e->dev);
    cudaMemcpyAsync(&v, &e->ctrl->argmax[b], 4, cudaMemcpyDeviceToHost, e->st);
    cudaStreamSynchronize(e->st);
    return v;
}

extern "C" float qb_last_loop_ms(qwen_model_t* m) {
    Engine* e = E_(m);
    return e ? e->last_ms : 0.f;
}

extern "C" int qb_prefill(qwen_model_t* m, const uint32_t* tokens, uint32_t n, int spec) {
    Engine* e = E_(m);
    if (!e || !tokens || n == 0 || n > (uint32_t)e->n_ctx) { set_err(-1, "qb_prefill: bad arguments"); return -1; }
    CK(cudaSetDevice(e->dev));
    spec = spec ? 1 : 0;
    // the whole prompt goes to the device once; every full chunk before the last is one
    // replay of a chunk graph, which takes its tokens from there at fwd_pos: chunks of
    // kPrefillW tokens while more than kPrefillW remain (one GPU), then of PREFILL_MAX_B
    CK(cudaMemcpyAsync(e->d_prompt, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, e->st));
    const uint32_t n_wide = e->tp_world == 1 && !e->fuse && !e->use_tc && n > (uint32_t)kPrefillW
                                ? (n - 1) / kPrefillW : 0;
    const uint32_t n_full = (n - n_wide * kPrefillW - 1) / PREFILL_MAX_B;   // 8-token chunks before the last
    if (n_wide && !e->g_prefill_w[spec] && capture(*e, &e->g_prefill_w[spec], record_prefill, spec | 2)) return -1;
    if (n_full && !e->g_prefill[spec] && capture(*e, &e->g_prefill[spec], record_prefill, spec)) return -1;
    CK(cudaEventRecord(e->ev0, e->st));
    CK(qb_launch(set_u32_kernel, dim3(1), dim3(1), 0, e->st, &e->ctrl->fwd_pos, 0u));
    for (uint32_t c = 0; c < n_wide; ++c) CK(cudaGraphLaunch(e->g_prefill_w[spec], e->st));
    for (uint32_t c = 0; c < n_full; ++c) CK(cudaGraphLaunch(e->g_prefill[spec], e->st));
    // the last chunk (1..8 tokens) with the output head: logits and argmax of its rows
    const uint32_t pos = n_wide * kPrefillW + n_full * PREFILL_MAX_B, lastB = n - pos;
    CK(cudaMemcpyAsync(e->ctrl->fwd_tok, e->d_prompt + pos, lastB * 4, cudaMemcpyDeviceToDevice, e->st));
    CK(qb_launch(set_u32_kernel, dim3(1), dim3(1), 0, e->st, &e->ctrl->fwd_pos, pos));
    if (fwd_backbone(*e, (int)lastB, 0, false, true)) return -1;
    if (spec) {
        CK(cudaMemcpyAsync(e->ctrl->mtp_tok, e->d_prompt + pos, lastB * 4, cudaMemcpyDeviceToDevice, e->st));
        CK(qb_launch(set_u32_kernel, dim3(1), dim3(1), 0, e->st, &e->ctrl->mtp_pos, pos));
        if (fwd_mtp(*e, (int)lastB, e->h_save, 0)) return -1;
    }
    CK(cudaEventRecord(e->ev1, e->st));
    // next cand0 = argmax of the last prompt token's logits
    CK(cudaMemcpyAsync(&e->ctrl->next_cand0, &e->ctrl->argmax[lastB - 1], 4, cudaMemcpyDeviceToDevice, e->st));
    CK(cudaMemcpyAsync(m->logits, e->logits + (size_t)(lastB - 1) * e->V, (size_t)e->V * 4, cudaMemcpyDeviceToHost,
                       e->st));
    CK(cudaMemcpyAsync(m->h_save, e->h_save, (size_t)lastB * e->E * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaMemcpyAsync(m->mtp_h, e->mtp_h, (size_t)e->E * 4, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    CK(cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1));
    m->pos = n;
    return 0;
}

extern "C" int qb_spec_generate(qwen_model_t* m, uint32_t n_predict, uint32_t n_spec, const uint32_t* forced,
                                uint32_t n_forced, uint32_t* out_tokens, uint32_t* out_j, uint32_t max_cycles,
                                uint32_t* n_cycles) {
    Engine* e = E_(m);
    if (!e || !out_tokens || m->pos == 0) { set_err(-1, "qb_spec_generate: bad arguments / no prefill"); return -1; }
    CK(cudaSetDevice(e->dev));
    const int k = (int)std::min<uint32_t>(n_spec, SPEC_MAX_B - 1);
    if (k < 1) { set_err(-1, "qb_spec_generate: n_spec must be >= 1"); return -1; }
    if (ensure_out_buffers(*e, n_predict + (uint32_t)k + 1, max_cycles, n_forced)) return -1;
    if (!e->g_cycle || e->g_cycle_k != k) {
        if (e->g_cycle) { cudaGraphExecDestroy(e->g_cycle); e->g_cycle = nullptr; }
        if (capture(*e, &e->g_cycle, record_cycle, k)) return -1;
        e->g_cycle_k = k;
        e->cycle_kernels = g_last_graph_kernels;
    }
    // loop state: P = pos - 1, counters reset, host mirror mtp_h is authoritative
    QbCtrl hc;
    CK(cudaMemcpyAsync(&hc, e->ctrl, sizeof hc, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    hc.P = m->pos - 1;
    hc.k = (uint32_t)k;
    hc.cycle = 0;
    hc.n_out = 0;
    hc.n_forced = n_forced;
    hc.cap_out = e->cap_out;
    hc.cap_j = max_cycles < e->cap_j ? max_cycles : e->cap_j;
    CK(cudaMemcpyAsync(e->ctrl, &hc, sizeof hc, cudaMemcpyHostToDevice, e->st));
    if (n_forced) CK(cudaMemcpyAsync(e->d_forced, forced, n_forced * 4, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->mtp_h, m->mtp_h, (size_t)e->E * 4, cudaMemcpyHostToDevice, e->st));

    uint32_t n_out = 0, cycles = 0;
    CK(cudaEventRecord(e->ev0, e->st));
    while (n_out < n_predict && cycles < max_cycles) {
        // never overshoot: each cycle emits at most k+1 tokens
        const uint32_t rem = n_predict - n_out;
        uint32_t batch = std::max<uint32_t>(1, rem / (uint32_t)(k + 1));
        batch = std::min(batch, max_cycles - cycles);
        const uint32_t P_now = m->pos - 1 + 0;   // updated below from the device
        (void)P_now;
        // context bound: every cycle advances P by at most k+1; verify writes P+1..P+k+1
        for (uint32_t i = 0; i < batch; ++i) CK(cudaGraphLaunch(e->g_cycle, e->st));
        cycles += batch;
        uint32_t dev_counts[2];
        CK(cudaMemcpyAsync(dev_counts, &e->ctrl->cycle, 8, cudaMemcpyDeviceToHost, e->st));   // cycle, n_out
        if (dev_sync(*e)) return -1;
        n_out = dev_counts[1];
        uint32_t P;
        CK(cudaMemcpyAsync(&P, &e->ctrl->P, 4, cudaMemcpyDeviceToHost, e->st));
        if (dev_sync(*e)) return -1;
        if (P + (uint32_t)k + 3 > (uint32_t)e->n_ctx) break;   // next cycle would pass n_ctx
    }
    CK(cudaEventRecord(e->ev1, e->st));
    CK(cudaEventSynchronize(e->ev1));
    cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
    const uint32_t n_copy = std::min(n_out, n_predict);
    CK(cudaMemcpyAsync(out_tokens, e->d_out_tok, (size_t)n_copy * 4, cudaMemcpyDeviceToHost, e->st));
    if (out_j)
        CK(cudaMemcpyAsync(out_j, e->d_out_j, (size_t)std::min(cycles, max_cycles) * 4, cudaMemcpyDeviceToHost, e->st));
    if (n_cycles) *n_cycles = cycles;
    // host mirrors: position, next logits (logits_b[j]), MTP hidden
    CK(cudaMemcpyAsync(&hc, e->ctrl, sizeof hc, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    m->pos = hc.P + 1;
    if (tp_fill_logits_row(*e, (int)hc.j)) return -1;
    CK(cudaMemcpyAsync(m->logits, e->logits + (size_t)hc.j * e->V, (size_t)e->V * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaMemcpyAsync(m->mtp_h, e->mtp_h, (size_t)e->E * 4, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    return (int)n_copy;
}

extern "C" int qb_greedy_generate(qwen_model_t* m, uint32_t n_predict, uint32_t* out_tokens) {
    Engine* e = E_(m);
    if (!e || !out_tokens || m->pos == 0) { set_err(-1, "qb_greedy_generate: bad arguments"); return -1; }
    if (n_predict == 0) return 0;
    CK(cudaSetDevice(e->dev));
    if (ensure_out_buffers(*e, n_predict + 1, 1, 1)) return -1;
    if (!e->g_greedy && capture(*e, &e->g_greedy, record_greedy, 0)) return -1;
    // token 0 = argmax(m->logits): the device argmax of the last forward
    QbCtrl hc;
    CK(cudaMemcpyAsync(&hc, e->ctrl, sizeof hc, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    hc.fwd_tok[0] = hc.next_cand0;
    hc.fwd_pos = m->pos;
    hc.greedy_n = 1;
    hc.cap_out = e->cap_out;
    CK(cudaMemcpyAsync(e->ctrl, &hc, sizeof hc, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->d_out_tok, &hc.next_cand0, 4, cudaMemcpyHostToDevice, e->st));
    uint32_t steps = n_predict - 1;
    if (m->pos + steps > (uint32_t)e->n_ctx) steps = (uint32_t)e->n_ctx - m->pos;
    CK(cudaEventRecord(e->ev0, e->st));
    for (uint32_t i = 0; i < steps; ++i) CK(cudaGraphLaunch(e->g_greedy, e->st));
    CK(cudaEventRecord(e->ev1, e->st));
    CK(cudaEventSynchronize(e->ev1));
    cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
    const uint32_t n = steps + 1;
    CK(cudaMemcpyAsync(out_tokens, e->d_out_tok, (size_t)n * 4, cudaMemcpyDeviceToHost, e->st));
    m->pos += steps;
    if (steps && tp_fill_logits_row(*e, 0)) return -1;
    CK(cudaMemcpyAsync(m->logits, e->logits, (size_t)e->V * 4, cudaMemcpyDeviceToHost, e->st));
    // keep next_cand0 = argmax of the last forward for a following call
    CK(cudaMemcpyAsync(&e->ctrl->next_cand0, &e->ctrl->argmax[0], 4, cudaMemcpyDeviceToDevice, e->st));
    if (dev_sync(*e)) return -1;
    return (int)n;
}

extern "C" int64_t qb_read_state(qwen_model_t* m, uint32_t il, int which, float* dst, int64_t max_floats) {
    Engine* e = E_(m);
    if (!e) return -1;
    cudaSetDevice(e->dev);
    const float* src = nullptr;
    size_t n = 0;
    uint32_t cur = 0;
    cudaMemcpyAsync(&cur, &e->ctrl->cur_slot, 4, cudaMemcpyDeviceToHost, e->st);
    cudaStreamSynchronize(e->st);
    if (il == e->d.n_layer) {
        if (which == 2) { src = e->mtp_k; n = e->kv_layer; }
        if (which == 3) { src = e->mtp_v; n = e->kv_layer; }
    } else if (il < e->d.n_layer) {
        const LayerW& l = e->L[il];
        if (l.rec && which == 0) { src = e->conv_slots + cur * e->conv_slot_stride + l.ridx * e->conv_layer; n = e->conv_layer; }
        if (l.rec && which == 1) { src = e->ssm_slots + cur * e->ssm_slot_stride + l.ridx * e->ssm_layer; n = e->ssm_layer; }
        if (!l.rec && which == 2) { src = e->kv_k + l.aidx * e->kv_layer; n = e->kv_layer; }
        if (!l.rec && which == 3) { src = e->kv_v + l.aidx * e->kv_layer; n = e->kv_layer; }
    }
    if (!src) return -1;
    if ((int64_t)n > max_floats) n = (size_t)max_floats;
    if (cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(e->st) != cudaSuccess) return -1;
    return (int64_t)n;
}

// New sequence: recurrent states and MTP hidden to zero, live slot 0, pos 0.
// KV entries need no clearing: positions >= pos are never read.
extern "C" int qb_reset(qwen_model_t* m) {
    Engine* e = E_(m);
    if (!e) return -1;
    CK(cudaSetDevice(e->dev));
    CK(cudaMemsetAsync(e->conv_slots, 0, std::max<size_t>(1, e->conv_slot_stride * kNSlot) * 4, e->st));
    CK(cudaMemsetAsync(e->ssm_slots, 0, std::max<size_t>(1, e->ssm_slot_stride * kNSlot) * 4, e->st));
    CK(cudaMemsetAsync(e->mtp_h, 0, (size_t)e->E * 4, e->st));
    set_u32_kernel<<<1, 1, 0, e->st>>>(&e->ctrl->cur_slot, 0u);
    CK(cudaGetLastError());
    if (dev_sync(*e)) return -1;
    memset(m->mtp_h, 0, (size_t)e->E * 4);
    m->pos = 0;
    return 0;
}

// ------------------------- multi-sequence decode ---------------------------------
// n_seq sequences share the weights; each gets its own recurrent slots, KV caches,
// control block and MTP hidden row (all zero), and one qb_seq_generate cycle runs
// drafts, verify and acceptance of all of them with one weight sweep per step:
// the MTP drafts at n_seq rows, the verify at n_seq (k + 1) rows, in QB_MAX_TOK-row
// GEMV chunks.
extern "C" int qb_seq_init(qwen_model_t* m, uint32_t n_seq) {
    Engine* e = E_(m);
    if (!e || n_seq < 1 || n_seq > QB_MAX_SEQ) { set_err(-1, "qb_seq_init: 1..%d sequences", QB_MAX_SEQ); return -1; }
    if (e->tp_world > 1 || e->fuse || e->use_tc) {
        set_err(-1, "qb_seq_init: multi-sequence decode runs on one GPU with the default GEMV paths");
        return -1;
    }
    CK(cudaSetDevice(e->dev));
    CK(cudaStreamSynchronize(e->st));
    select_seq(*e, 0);
    drop_graphs(*e);
    int na = 0;
    for (const LayerW& l : e->L) na += l.rec ? 0 : 1;
    const size_t conv1 = std::max<size_t>(1, e->conv_slot_stride * kNSlot), ssm1 = std::max<size_t>(1, e->ssm_slot_stride * kNSlot);
    const size_t kv1 = std::max<size_t>(1, e->kv_layer * (size_t)na), mtp1 = e->kv_layer, h1 = (size_t)e->E;
    const size_t q_rows = (size_t)e->d.n_head * QB_MAX_TOK * qb_attn_max_chunks(e->n_ctx);
    const size_t n_part = std::max<size_t>(n_seq, kAttnGroups);   // sequences, or prefill query groups
    // the new arrays first: if one does not fit, the model keeps its current sequences
    const size_t S = n_seq;
    const size_t sizes[10] = {S * conv1 * 4, S * ssm1 * 4,   S * kv1 * 4,  S * kv1 * 4,
                              S * mtp1 * 4,  S * mtp1 * 4,   S * h1 * 4,   S * sizeof(QbCtrl),
                              n_part * q_rows * e->d.head_dim * 4, n_part * q_rows * sizeof(float2)};
    void* fresh[10] = {};
    for (int i = 0; i < 10; ++i)
        if (!(fresh[i] = e->dalloc(sizes[i]))) {
            for (int j = 0; j < i; ++j) e->dfree(fresh[j]);
            set_err(-2, "qb_seq_init: state for %u sequences does not fit (%zu bytes more)", n_seq, sizes[i]);
            return -1;
        }
    void* olds[] = {e->conv_base, e->ssm_base, e->kv_k_base, e->kv_v_base, e->mtp_k_base, e->mtp_v_base,
                    e->mtp_h_base, e->ctrl_base, e->attn_po, e->attn_pml};
    for (void* p : olds) e->dfree(p);
    e->conv_base = (float*)fresh[0];
    e->ssm_base = (float*)fresh[1];
    e->kv_k_base = (float*)fresh[2];
    e->kv_v_base = (float*)fresh[3];
    e->mtp_k_base = (float*)fresh[4];
    e->mtp_v_base = (float*)fresh[5];
    e->mtp_h_base = (float*)fresh[6];
    e->ctrl_base = (QbCtrl*)fresh[7];
    e->attn_po = (float*)fresh[8];
    e->attn_pml = (float2*)fresh[9];
    CK(cudaMemsetAsync(e->conv_base, 0, S * conv1 * 4, e->st));
    CK(cudaMemsetAsync(e->ssm_base, 0, S * ssm1 * 4, e->st));
    CK(cudaMemsetAsync(e->mtp_h_base, 0, S * h1 * 4, e->st));
    CK(cudaMemsetAsync(e->ctrl_base, 0, S * sizeof(QbCtrl), e->st));
    const char* tcw_env = getenv("QB_TCW");   // QB_TCW=0: wide verifies in 8-row mma.sync chunks only
    if (n_seq * SPEC_MAX_B > QB_MAX_TOK && !(tcw_env && tcw_env[0] == '0') && enable_tcw(*e)) return -1;
    e->seq_conv = (long long)conv1;
    e->seq_ssm = (long long)ssm1;
    e->seq_kv = (long long)kv1;
    e->seq_mtpkv = (long long)mtp1;
    e->n_seq = (int)n_seq;
    e->cur_seq = -1;
    select_seq(*e, 0);
    e->seq_pos.assign(n_seq, 0u);
    // per-sequence output buffers are sized on the next call
    if (e->d_out_tok) cudaFree(e->d_out_tok);
    if (e->d_out_j) cudaFree(e->d_out_j);
    e->d_out_tok = e->d_out_j = nullptr;
    e->cap_out = e->cap_j = 0;
    if (dev_sync(*e)) return -1;
    memset(m->mtp_h, 0, (size_t)e->E * 4);
    m->pos = 0;
    return 0;
}

extern "C" int qb_enable_wide(qwen_model_t* m) {
    Engine* e = E_(m);
    if (!e) { set_err(-1, "qb_enable_wide: no model"); return -1; }
    CK(cudaSetDevice(e->dev));
    return enable_tcw(*e);
}

extern "C" int qb_seq_prefill(qwen_model_t* m, uint32_t seq, const uint32_t* tokens, uint32_t n) {
    Engine* e = E_(m);
    if (!e || seq >= (uint32_t)e->n_seq) { set_err(-1, "qb_seq_prefill: no sequence %u", seq); return -1; }
    CK(cudaSetDevice(e->dev));
    select_seq(*e, (int)seq);
    if (qb_prefill(m, tokens, n, 1)) return -1;
    e->seq_pos[seq] = n;
    return 0;
}

extern "C" int qb_seq_generate(qwen_model_t* m, uint32_t n_cycles, uint32_t n_spec, const uint32_t* forced,
                               uint32_t n_forced, uint32_t* out_tokens, uint32_t cap, uint32_t* out_counts,
                               uint32_t* out_j) {
    Engine* e = E_(m);
    if (!e || !out_tokens || !out_counts || cap == 0) { set_err(-1, "qb_seq_generate: bad arguments"); return -1; }
    CK(cudaSetDevice(e->dev));
    const int S = e->n_seq;
    const int k = (int)std::min<uint32_t>(n_spec, SPEC_MAX_B - 1);
    if (k < 1 || S * (k + 1) > QB_WIDE) {
        set_err(-1, "qb_seq_generate: n_spec must be >= 1 and n_seq (n_spec + 1) <= %d", QB_WIDE);
        return -1;
    }
    for (int s = 0; s < S; ++s)
        if (e->seq_pos[s] == 0) { set_err(-1, "qb_seq_generate: sequence %d has no prefill", s); return -1; }
    if (ensure_out_buffers(*e, cap + (uint32_t)k + 1, n_cycles, n_forced)) return -1;
    select_seq(*e, 0);
    if (!e->g_mcycle || e->g_mcycle_k != k) {
        if (e->g_mcycle) { cudaGraphExecDestroy(e->g_mcycle); e->g_mcycle = nullptr; }
        e->ms_S = S;
        const int r = capture(*e, &e->g_mcycle, record_cycle, k);
        e->ms_S = 1;
        if (r) return -1;
        e->g_mcycle_k = k;
        e->mcycle_kernels = g_last_graph_kernels;
    }
    // loop state of every sequence: P = tokens consumed - 1, counters reset
    std::vector<QbCtrl> hc((size_t)S);
    CK(cudaMemcpyAsync(hc.data(), e->ctrl_base, S * sizeof(QbCtrl), cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    for (int s = 0; s < S; ++s) {
        hc[s].P = e->seq_pos[s] - 1;
        hc[s].k = (uint32_t)k;
        hc[s].cycle = 0;
        hc[s].n_out = 0;
        hc[s].n_forced = n_forced;
        hc[s].cap_out = std::min(cap, e->cap_out);
        hc[s].cap_j = std::min(n_cycles, e->cap_j);
    }
    CK(cudaMemcpyAsync(e->ctrl_base, hc.data(), S * sizeof(QbCtrl), cudaMemcpyHostToDevice, e->st));
    if (n_forced) CK(cudaMemcpyAsync(e->d_forced, forced, n_forced * 4, cudaMemcpyHostToDevice, e->st));
    uint32_t cycles = 0;
    CK(cudaEventRecord(e->ev0, e->st));
    while (cycles < n_cycles) {
        // every cycle moves a sequence by at most k + 1 positions; verify writes P+1..P+k+1
        uint32_t Pmax = 0;
        for (int s = 0; s < S; ++s) Pmax = std::max(Pmax, hc[s].P);
        const uint32_t room = (uint32_t)e->n_ctx > Pmax + (uint32_t)k + 2 ? ((uint32_t)e->n_ctx - Pmax - k - 2) / (k + 1) : 0;
        const uint32_t batch = std::min(std::min(n_cycles - cycles, 32u), room);
        if (batch == 0) break;
        for (uint32_t i = 0; i < batch; ++i) CK(cudaGraphLaunch(e->g_mcycle, e->st));
        cycles += batch;
        CK(cudaMemcpyAsync(hc.data(), e->ctrl_base, S * sizeof(QbCtrl), cudaMemcpyDeviceToHost, e->st));
        if (dev_sync(*e)) return -1;
    }
    CK(cudaEventRecord(e->ev1, e->st));
    CK(cudaEventSynchronize(e->ev1));
    cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
    for (int s = 0; s < S; ++s) {
        out_counts[s] = std::min(hc[s].n_out, cap);
        CK(cudaMemcpyAsync(out_tokens + (size_t)s * cap, e->d_out_tok + (size_t)s * e->cap_out, (size_t)out_counts[s] * 4,
                           cudaMemcpyDeviceToHost, e->st));
        if (out_j)
            CK(cudaMemcpyAsync(out_j + (size_t)s * n_cycles, e->d_out_j + (size_t)s * e->cap_j,
                               (size_t)std::min(cycles, hc[s].cap_j) * 4, cudaMemcpyDeviceToHost, e->st));
        e->seq_pos[s] = hc[s].P + 1;
    }
    if (dev_sync(*e)) return -1;
    m->pos = e->seq_pos[0];
    return (int)cycles;
}

namespace {
size_t mat_bytes(const DevMat& w) { return w.bytes_all; }

int record_verify(Engine& e, int B) { return fwd_backbone(e, B, 1); }
int record_draft(Engine& e, int) { return fwd_mtp(e, 1, e.mtp_h, 1); }
}  // namespace

// Device timing of one component, averaged over `iters` runs, CUDA events on
// the engine stream.  what: 0 verify forward of `arg` tokens (64 layers +
// head, graph replay), 1 fused FFN gate+up GEMV with N = arg rotating over
// all layers, 2 one MTP draft with logits, 3 output-head GEMV with N = arg,
// 5 / 6 / 7 the FFN down / mixer out-projection / mixer in-projection GEMV
// with N = arg rotating over all layers, as the forward launches them.
// *bytes = algorithmic bytes of one run (GGUF weight bytes + activations and
// states read/written once).  Mutates KV / recurrent state: call last.
extern "C" float qb_bench(qwen_model_t* m, int what, uint32_t arg, uint32_t iters, double* bytes) {
    Engine* e = E_(m);
    if (!e || iters == 0) return -1.f;
    if (cudaSetDevice(e->dev) != cudaSuccess) return -1.f;
    const qwen_dims_t& d = e->d;
    double b = 0;
    float ms = 0.f;
    cudaGraphExec_t ge = nullptr;
    if (what == 0 || what == 2) {
        if (what == 0 && (arg < 1 || arg > SPEC_MAX_B)) return -1.f;
        if (capture(*e, &ge, what == 0 ? record_verify : record_draft, (int)arg)) return -1.f;
        cudaGraphLaunch(ge, e->st);   // warm
        cudaEventRecord(e->ev0, e->st);
        for (uint32_t i = 0; i < iters; ++i) cudaGraphLaunch(ge, e->st);
        cudaEventRecord(e->ev1, e->st);
        cudaEventSynchronize(e->ev1);
        cudaEventElapsedTime(&ms, e->ev0, e->ev1);
        cudaGraphExecDestroy(ge);
        if (what == 0) {
            for (const LayerW& l : e->L) {
                b += mat_bytes(l.ffn_gate) + mat_bytes(l.ffn_up) + mat_bytes(l.ffn_down);
                if (l.rec) b += mat_bytes(l.wqkv) + mat_bytes(l.wgate) + mat_bytes(l.wbeta) + mat_bytes(l.walpha) + mat_bytes(l.ssm_out);
                else b += mat_bytes(l.q) + mat_bytes(l.k) + mat_bytes(l.v) + mat_bytes(l.o);
            }
            b += mat_bytes(e->output);
            b += 2.0 * e->ssm_slot_stride * 4 + 2.0 * e->conv_slot_stride * 4;   // states read + written once
            uint32_t pos = 0;
            cudaMemcpyAsync(&pos, &e->ctrl->fwd_pos, 4, cudaMemcpyDeviceToHost, e->st);
            cudaStreamSynchronize(e->st);
            b += (double)d.n_attn_layer * (pos + arg) * 2.0 * d.n_kv_head * d.head_dim * 4;   // KV read once
        } else {
            const LayerW& l = e->mtp;
            b = mat_bytes(e->eh_proj) + mat_bytes(l.q) + mat_bytes(l.k) + mat_bytes(l.v) + mat_bytes(l.o) +
                mat_bytes(l.ffn_gate) + mat_bytes(l.ffn_up) + mat_bytes(l.ffn_down) + mat_bytes(e->output);
        }
    } else if (what == 1 || what == 3 || (what >= 5 && what <= 8)) {
        if (arg < 1 || arg > QB_MAX_TOK) return -1.f;
        // one graph of the launches (all layers except for the head), replayed: no host launch gaps
        const int nl = what != 3 ? (int)e->L.size() : 1;
        struct Rec {
            static int go(Engine& en, int packed) {
                const int wh = packed & 0xFF, a = (packed >> 8) & 0xFF, nlay = packed >> 16;
                for (int li = 0; li < nlay; ++li) {
                    const LayerW& ly = en.L[li];
                    if (wh == 5) {
                        fresh_input(en);
                        if (residual_gemv(en, &ly.ffn_down, en.bx, en.F_loc, a, nullptr)) return -1;
                    } else if (wh == 6) {
                        fresh_input(en);
                        const int K = ly.rec ? en.nv_loc * (int)en.d.head_v_dim : en.nh_loc * (int)en.d.head_dim;
                        if (residual_gemv(en, ly.rec ? &ly.ssm_out : &ly.o, en.bx, K, a, nullptr)) return -1;
                    } else if (wh == 7) {
                        fresh_input(en);
                        if (ly.rec) {
                            const DevMat* m4[4] = {&ly.wqkv, &ly.wgate, &ly.wbeta, &ly.walpha};
                            float* o4[4] = {en.qkv, en.z, en.beta, en.alpha};
                            const long long ld4[4] = {en.ld_qkv, (long long)en.d.d_inner, 256, 256};
                            if (gemv_group(en, m4, o4, ld4, 4, en.E, a, 0)) return -1;
                        } else {
                            const DevMat* m3[3] = {&ly.q, &ly.k, &ly.v};
                            float* o3[3] = {en.qbuf, en.kvbuf, en.kvbuf + ly.k.rows_all};
                            const long long ld3[3] = {2LL * en.d.n_head * en.d.head_dim,
                                                      2LL * en.d.n_kv_head * en.d.head_dim,
                                                      2LL * en.d.n_kv_head * en.d.head_dim};
                            if (gemv_group(en, m3, o3, ld3, 3, en.E, a, 0)) return -1;
                        }
                    } else if (wh == 8) {
                        // one FFN up matrix alone (the 17408 x 5120 IQ4_XS micro)
                        fresh_input(en);
                        const DevMat* m1[1] = {&ly.ffn_up};
                        float* o1[1] = {en.up};
                        const long long ld1[1] = {en.F};
                        if (!ly.ffn_up.w || gemv_group(en, m1, o1, ld1, 1, en.E, a, 0)) return -1;
                    } else if (wh == 1) {
                        // the FFN gate / up launch as the forward runs it
                        const LayerW& l = en.L[li];
                        if (l.gu.w) {
                            const QbEpi sw{QB_EPI_SWIGLU, nullptr, nullptr, en.act, en.F, en.xb_alt,
                                           xp_needs(en, {&l.ffn_down}, a)};
                            const DevMat* m1[1] = {&l.gu};
                            float* o1[1] = {en.act};
                            const long long ld1[1] = {en.F};
                            if (gemv_group(en, m1, o1, ld1, 1, en.E, a, 0, &sw)) return -1;
                        } else {
                            const DevMat* m2[2] = {&l.ffn_gate, &l.ffn_up};
                            float* o2[2] = {en.gate, en.up};
                            const long long ld2[2] = {en.F, en.F};
                            if (gemv_group(en, m2, o2, ld2, 2, en.E, a, 0)) return -1;
                        }
                    } else {
                        const DevMat* m1[1] = {&en.output};
                        float* o1[1] = {en.logits};
                        const long long ld1[1] = {en.V};
                        if (gemv_group(en, m1, o1, ld1, 1, en.E, a, 0, nullptr, TP_GATHER)) return -1;
                    }
                }
                return 0;
            }
        };
        if (capture(*e, &ge, Rec::go, what | ((int)arg << 8) | (nl << 16))) return -1.f;
        cudaGraphLaunch(ge, e->st);
        cudaEventRecord(e->ev0, e->st);
        for (uint32_t i = 0; i < iters; ++i) cudaGraphLaunch(ge, e->st);
        cudaEventRecord(e->ev1, e->st);
        cudaEventSynchronize(e->ev1);
        cudaEventElapsedTime(&ms, e->ev0, e->ev1);
        cudaGraphExecDestroy(ge);
        iters *= (uint32_t)nl;
        const LayerW& l0 = e->L[0];
        if (what == 1 || what == 3 || what == 8) {
            b = what == 1   ? (double)(mat_bytes(l0.ffn_gate) + mat_bytes(l0.ffn_up))
                : what == 8 ? (double)mat_bytes(l0.ffn_up)
                            : (double)mat_bytes(e->output);
            b += (double)arg * e->E * 4 + (double)arg * (what == 1 ? 2.0 * e->F : what == 8 ? e->F : e->V) * 4;
        } else {
            for (const LayerW& l : e->L) {   // the average launch over the layers
                if (what == 5) b += mat_bytes(l.ffn_down);
                else if (what == 6) b += mat_bytes(l.rec ? l.ssm_out : l.o);
                else if (l.rec) b += mat_bytes(l.wqkv) + mat_bytes(l.wgate) + mat_bytes(l.wbeta) + mat_bytes(l.walpha);
                else b += mat_bytes(l.q) + mat_bytes(l.k) + mat_bytes(l.v);
            }
            b /= (double)nl;
        }
    } else if (what == 10) {
        // one FFN up matrix at N = arg (1..32), rotated over all layers, on the wide tcgen05
        // GEMM; the tcgen05 tile copies of those matrices are made on first use
        if (arg < 1 || arg > QB_TCW_TOK || e->tp_world > 1) return -1.f;
        const int nl = (int)e->L.size();
        for (int li = 0; li < nl; ++li)
            if (ensure_w_tc(*e, e->L[li].ffn_up)) return -1.f;
        if (!e->xb16.xtc16) {
            e->xb16.xtc16 = (uint8_t*)e->dalloc(qb_xtc16_bytes(e->E));
            e->xb16.xtc32 = (uint8_t*)e->dalloc(qb_xtc32_bytes(e->E));
            e->xb16.xqscale = (float*)e->dalloc((size_t)QB_TCW_TOK * (e->E / 256) * 4);
            if (!e->xb16.xtc16 || !e->xb16.xtc32 || !e->xb16.xqscale) return -1.f;
        }
        // input: arg rows of the FFN activation buffer (any finite values), prepared once
        const QbXIn in{e->act, e->E, nullptr, e->E};
        const int xw = arg <= QB_TC16_TOK ? QB_XP_TC16 : QB_XP_TC32;
        if (qb_xprep(&in, 1, (int)arg, e->eps, e->xb16, xw, e->st) != cudaSuccess) return -1.f;
        struct Rec9 {
            static int go(Engine& en, int a) {
                for (const LayerW& ly : en.L) {
                    QbQSeg seg;
                    seg.w = ly.ffn_up.w_tc;
                    seg.out = en.logits;   // [a][F] rows of the logits buffer
                    seg.ldo = en.F;
                    seg.rows = ly.ffn_up.rows;
                    CK(qb_qmv_tcw(&seg, 1, en.E, a, en.xb16, 0, 0, 1 << 30, en.work, en.st));
                }
                return 0;
            }
        };
        if (capture(*e, &ge, Rec9::go, (int)arg)) return -1.f;
        cudaGraphLaunch(ge, e->st);
        cudaEventRecord(e->ev0, e->st);
        for (uint32_t i = 0; i < iters; ++i) cudaGraphLaunch(ge, e->st);
        cudaEventRecord(e->ev1, e->st);
        cudaEventSynchronize(e->ev1);
        cudaEventElapsedTime(&ms, e->ev0, e->ev1);
        cudaGraphExecDestroy(ge);
        iters *= (uint32_t)nl;
        b = (double)mat_bytes(e->L[0].ffn_up) + (double)arg * e->E * 4 + (double)arg * e->F * 4;
    } else if (what == 4) {
        // kernels launched per speculative cycle (nodes of the captured cycle graph)
        if (bytes) *bytes = 0;
        return (float)e->cycle_kernels;
    } else {
        return -1.f;
    }
    if (cudaGetLastError() != cudaSuccess) return -1.f;
    if (bytes) *bytes = b;
    return ms / (float)iters;
}

// Copy an internal activation buffer to host (debugging / layer-level parity).
extern "C" int64_t qb_read_buffer(qwen_model_t* m, int id, float* dst, int64_t max_floats) {
    Engine* e = E_(m);
    if (!e) return -1;
    cudaSetDevice(e->dev);
    const qwen_dims_t& d = e->d;
    const float* src = nullptr;
    size_t n = 0;
    const size_t T8 = QB_MAX_TOK;
    switch (id) {
    case 0: src = e->bx; n = T8 * e->E; break;
    case 1: src = e->qkv; n = T8 * e->ld_qkv; break;
    case 2: src = e->qkvc; n = T8 * e->ld_qkv; break;
    case 3: src = e->z; n = T8 * d.d_inner; break;
    case 4: src = e->beta; n = T8 * 256; break;
    case 5: src = e->alpha; n = T8 * 256; break;
    case 6: src = e->o; n = T8 * d.d_inner; break;
    case 7: src = e->y; n = T8 * d.d_inner; break;
    case 8: src = e->qbuf; n = T8 * 2 * d.n_head * d.head_dim; break;
    case 9: src = e->kvbuf; n = T8 * 2 * d.n_kv_head * d.head_dim; break;
    case 10: src = e->attn_o; n = T8 * d.n_head * d.head_dim; break;
    case 11: src = e->gate; n = T8 * e->F; break;
    case 12: src = e->up; n = T8 * e->F; break;
    case 13: src = e->act; n = T8 * e->F; break;
    case 14: src = e->emb; n = T8 * e->E; break;
    case 15: src = e->mtp_x; n = T8 * e->E; break;
    case 16: src = e->h_save; n = T8 * e->E; break;
    default: return -1;
    }
    if ((int64_t)n > max_floats) n = (size_t)max_floats;
    if (cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) return -1;
    if (cudaStreamSynchronize(e->st) != cudaSuccess) return -1;
    return (int64_t)n;
}

// ============================ C API: kernels.h ====================================
// Host-pointer GEMV and element-wise ops.  Weights are uploaded + repacked on
// first use and cached per device, keyed by (device, W->data, type, shape).

namespace {
struct WKey {
    int dev;
    const void* p;
    int type;
    uint64_t ne0, ne1;
    bool operator==(const WKey& o) const { return dev == o.dev && p == o.p && type == o.type && ne0 == o.ne0 && ne1 == o.ne1; }
};
struct WKeyHash {
    size_t operator()(const WKey& k) const {
        return std::hash<const void*>()(k.p) ^ (std::hash<uint64_t>()(k.ne0 * 131 + k.ne1) << 1) ^ (size_t)k.type ^ ((size_t)k.dev << 7);
    }
};
struct Scratch {
    cudaStream_t st = nullptr;
    float *x = nullptr, *out = nullptr;
    size_t x_cap = 0, out_cap = 0;
    QbXBuf xb{};
    size_t k_cap = 0;
    unsigned long long* keys = nullptr;
    uint32_t* am = nullptr;
    QbQmvWork work{};
};
std::mutex g_mu;
constexpr int QB_GEMV_MULTI_MAX = 8;   // src/kernels.c:657 (GEMV_MULTI_MAX)
// host GEMV API: IQ4_XS at n <= 4 on tcgen05 (QB_TC=1); default: int8 mma.sync
bool host_tc() {
    static const bool on = [] {
        const char* tc = getenv("QB_TC");
        return tc && tc[0] == '1';
    }();
    return on;
}
std::unordered_map<WKey, DevMat, WKeyHash> g_wcache;
std::unordered_map<int, Scratch> g_scratch;

int scratch_get(Scratch*& s, size_t x_floats, size_t out_floats, int K) {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    s = &g_scratch[dev];
    if (!s->st) {
        CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    }
    if (x_floats > s->x_cap) {
        if (s->x) cudaFree(s->x);
        s->x_cap = std::max<size_t>(x_floats, 1 << 16);
        CK(cudaMalloc(&s->x, s->x_cap * 4));
    }
    if (out_floats > s->out_cap) {
        if (s->out) cudaFree(s->out);
        s->out_cap = std::max<size_t>(out_floats, 1 << 16);
        CK(cudaMalloc(&s->out, s->out_cap * 4));
    }
    if ((size_t)K > s->k_cap) {
        if (s->xb.xfrag) cudaFree(s->xb.xfrag);
        if (s->xb.xscale) cudaFree(s->xb.xscale);
        if (s->xb.xsum) cudaFree(s->xb.xsum);
        if (s->xb.xq) cudaFree(s->xb.xq);
        if (s->xb.xqscale) cudaFree(s->xb.xqscale);
        if (s->xb.xtc) cudaFree(s->xb.xtc);
        if (s->xb.xtc16) cudaFree(s->xb.xtc16);
        if (s->xb.xtc32) cudaFree(s->xb.xtc32);
        s->k_cap = std::max<size_t>((size_t)K, 4096);
        const int kc = (int)((s->k_cap + 255) / 256 * 256);
        CK(cudaMalloc(&s->xb.xfrag, qb_xfrag_bytes(kc)));
        CK(cudaMemset(s->xb.xfrag, 0, qb_xfrag_bytes(kc)));
        CK(cudaMalloc(&s->xb.xq, qb_xq_bytes(kc)));
        CK(cudaMemset(s->xb.xq, 0, qb_xq_bytes(kc)));
        CK(cudaMalloc(&s->xb.xscale, QB_MAX_TOK * (kc / 256) * 4));
        CK(cudaMalloc(&s->xb.xqscale, QB_TCW_TOK * (kc / 256) * 4));   // the 32-token path's rows too
        CK(cudaMalloc(&s->xb.xtc16, qb_xtc16_bytes(kc)));
        CK(cudaMemset(s->xb.xtc16, 0, qb_xtc16_bytes(kc)));
        CK(cudaMalloc(&s->xb.xtc32, qb_xtc32_bytes(kc)));
        CK(cudaMemset(s->xb.xtc32, 0, qb_xtc32_bytes(kc)));
        CK(cudaMalloc(&s->xb.xtc, qb_xtc_bytes(kc)));
        CK(cudaMemset(s->xb.xtc, 0, qb_xtc_bytes(kc)));
        CK(cudaMalloc(&s->xb.xsum, QB_MAX_TOK * (kc / 32) * 4));
    }
    if (!s->keys) {
        CK(cudaMalloc(&s->keys, QB_MAX_TOK * sizeof(unsigned long long)));
        CK(cudaMalloc(&s->am, QB_MAX_TOK * 4));
    }
    return 0;
}

int scratch_work(Scratch* s, int rows) {
    const int pairs = (rows + 31) / 32 + 1;
    if (pairs > s->work.max_pairs) {
        qb_qmv_work_free(s->work);
        CK(qb_qmv_work_alloc(s->work, std::max(pairs, 8192)));
    }
    return 0;
}

// FNV-1a over 64 evenly spaced 16-byte windows plus both ends of the weight
// bytes.  The device copy is keyed by (pointer, type, shape) as the reference
// hands out stable mmap pointers; the fingerprint catches a caller that
// reuses an address for different weights (freed and reallocated buffers).
uint64_t weight_fingerprint(const uint8_t* p, size_t n) {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](size_t off, size_t len) {
        for (size_t i = 0; i < len && off + i < n; ++i) h = (h ^ p[off + i]) * 1099511628211ull;
    };
    mix(0, 64);
    for (int k = 0; k < 64; ++k) mix(n / 64 * (size_t)k, 16);
    if (n > 64) mix(n - 64, 64);
    return h;
}

int wcache_get(const gguf_tensor_info_t* W, const DevMat*& out) {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    const WKey key{dev, W->data, (int)W->type, W->ne[0], W->ne[1]};
    const size_t src_bytes = gguf_row_bytes((int)W->type, W->ne[0]) * W->ne[1];
    const uint64_t fp = src_bytes ? weight_fingerprint((const uint8_t*)W->data, src_bytes) : 0;
    auto it = g_wcache.find(key);
    if (it != g_wcache.end()) {
        if (it->second.fingerprint == fp) { out = &it->second; return 0; }
        cudaFree(it->second.w);   // same address, different weights: replace the device copy
        if (it->second.w_tc) cudaFree(it->second.w_tc);
        g_wcache.erase(it);
    }
    DevMat m;
    m.type = (int)W->type;
    m.K = (int)W->ne[0];
    m.rows = (int)W->ne[1];
    m.fingerprint = fp;
    if (!src_bytes || (m.type != QB_F32 && m.K % 256)) { set_err(-1, "gemv: unsupported tensor type %d / ne0 %llu", m.type, (unsigned long long)W->ne[0]); return -1; }
    if (m.type == QB_F32) {
        CK(cudaMalloc(&m.w, src_bytes));
        CK(cudaMemcpy(m.w, W->data, src_bytes, cudaMemcpyHostToDevice));
        CK(cudaDeviceSynchronize());   // the DMA from pageable memory may still be in flight
    } else {
        void* tmp = nullptr;
        CK(cudaMalloc(&tmp, src_bytes));
        CK(cudaMemcpy(tmp, W->data, src_bytes, cudaMemcpyHostToDevice));
        CK(cudaMalloc(&m.w, qb_repacked_bytes(m.type, m.rows, m.K)));
        CK(qb_repack(m.type, tmp, m.rows, m.K, m.w, 0));
        if (m.type == QB_IQ4_XS && host_tc()) {
            CK(cudaMalloc(&m.w_tc, qb_repacked_bytes_tc(m.rows, m.K)));
            CK(qb_repack_tc(tmp, m.rows, m.K, m.w_tc, 0));
        }
        CK(cudaDeviceSynchronize());
        cudaFree(tmp);
    }
    out = &(g_wcache[key] = m);
    return 0;
}

// the tcgen05 tile layout of an IQ4_XS matrix of the host API, repacked from
// the caller's blocks on first use (the wide tcgen05 path reads it)
int wcache_tc(const gguf_tensor_info_t* W, const DevMat* M) {
    if (M->w_tc) return 0;
    const size_t src_bytes = gguf_row_bytes((int)W->type, W->ne[0]) * W->ne[1];
    void* tmp = nullptr;
    void* dst = nullptr;
    CK(cudaMalloc(&tmp, src_bytes));
    CK(cudaMemcpy(tmp, W->data, src_bytes, cudaMemcpyHostToDevice));
    CK(cudaMalloc(&dst, qb_repacked_bytes_tc(M->rows, M->K)));
    CK(qb_repack_tc(tmp, M->rows, M->K, dst, 0));
    CK(cudaDeviceSynchronize());
    cudaFree(tmp);
    const_cast<DevMat*>(M)->w_tc = dst;
    return 0;
}

// out_i[t][r] = W_i x[t] for the n_mat matrices (all reading the same x), rows
// [r0, r1) of each (r1 clamped to its rows), t < n, host x / outs.  One
// dispatch: per chunk of vectors (QB_MAX_TOK, or QB_TCW_TOK for IQ4_XS above
// QB_MAX_TOK vectors), one host-to-device copy of x, one activation prep
// covering every format and width, one GEMV launch per matrix queued back to
// back (each the launch a single-matrix call makes, so the results are
// bit-identical to separate calls, as src/kernels.c:650-655 promises for the
// CPU), the device-to-host copies, one synchronisation.
int gemv_multi_host(const gguf_tensor_info_t* const* Ws, int n_mat, const float* x, uint64_t ldx, int n,
                    float* const* outs, const uint64_t* ldos, uint64_t r0, uint64_t r1) {
    if (!Ws || !x || !outs || !ldos || n < 1 || n_mat < 1 || n_mat > QB_GEMV_MULTI_MAX) {
        set_err(-1, "gemv: bad arguments (n %d, n_mat %d, at most %d matrices)", n, n_mat, QB_GEMV_MULTI_MAX);
        return -1;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    const DevMat* M[QB_GEMV_MULTI_MAX];
    uint64_t lo[QB_GEMV_MULTI_MAX], hi[QB_GEMV_MULTI_MAX];
    int Kmax = 0;
    int need = 0;
    for (int i = 0; i < n_mat; ++i) {
        if (!Ws[i] || !outs[i]) { set_err(-1, "gemv: null matrix or output %d", i); return -1; }
        if (wcache_get(Ws[i], M[i])) return -1;
        Kmax = std::max(Kmax, M[i]->K);
        hi[i] = std::min<uint64_t>(r1, (uint64_t)M[i]->rows);
        lo[i] = std::min(r0, hi[i]);
    }
    if (ldx < (uint64_t)Kmax) { set_err(-1, "gemv: ldx %llu < ne0 %d", (unsigned long long)ldx, Kmax); return -1; }
    // more vectors than one mma.sync sweep takes: IQ4_XS matrices run 32 per sweep on
    // tcgen05 (qb_qmv_tcw), the others 8 per sweep.  The path is a property of the
    // matrix and n alone, so a matrix gives the same bits here as in its own
    // gemv_batch call.
    bool wide_of[QB_GEMV_MULTI_MAX];
    for (int i = 0; i < n_mat; ++i) {
        wide_of[i] = n > QB_MAX_TOK && M[i]->type == QB_IQ4_XS;
        if (wide_of[i] && wcache_tc(Ws[i], M[i])) return -1;
    }
    Scratch* s = nullptr;
    for (int pass = 0; pass < 2; ++pass) {   // pass 0: 8-vector chunks, pass 1: 32-vector chunks
        const bool wide = pass == 1;
        bool any = false;
        size_t of = 0;
        for (int i = 0; i < n_mat; ++i)
            if (wide_of[i] == wide) {
                any = true;
                of += (size_t)std::min(n, wide ? QB_TCW_TOK : QB_MAX_TOK) * M[i]->rows;
            }
        if (!any) continue;
        const int chunk = wide ? QB_TCW_TOK : QB_MAX_TOK;
        for (int t0 = 0; t0 < n; t0 += chunk) {
            const int nn = std::min(chunk, n - t0);
            if (scratch_get(s, (size_t)nn * Kmax, of, Kmax)) return -1;
            CK(cudaMemcpy2DAsync(s->x, (size_t)Kmax * 4, x + (size_t)t0 * ldx, ldx * 4, (size_t)Kmax * 4, nn,
                                 cudaMemcpyHostToDevice, s->st));
            need = 0;
            for (int i = 0; i < n_mat; ++i) {
                if (wide_of[i] != wide || M[i]->type == QB_F32) continue;
                const bool tc = M[i]->w_tc && nn <= 4 && host_tc();
                need |= wide ? (nn <= QB_TC16_TOK ? QB_XP_TC16 : QB_XP_TC32) : qb_xprep_needs(M[i]->type, nn, tc ? 1 : 0);
                if (scratch_work(s, M[i]->rows)) return -1;
            }
            if (need) {
                QbXIn in{s->x, Kmax, nullptr, Kmax};
                CK(qb_xprep(&in, 1, nn, 1e-6f, s->xb, need, s->st));
            }
            float* o = s->out;
            for (int i = 0; i < n_mat; ++i) {
                if (wide_of[i] != wide) continue;
                const DevMat* W = M[i];
                const int K = W->K;
                const uint64_t a = lo[i], b = hi[i];
                if (a < b) {
                    const int t_lo = (int)(a / (2 * QB_TILE)) * 2;   // start on a tile pair
                    if (W->type == QB_F32) {
                        CK(qb_qmv_f32((const float*)W->w, W->rows, K, s->x, Kmax, nn, o, W->rows, 0, (int)a, (int)b,
                                      s->st));
                    } else if (wide || (W->w_tc && nn <= 4 && host_tc())) {
                        const int T0 = (int)(a / 128);   // start on a 128-row tile
                        QbQSeg seg;
                        seg.w = (const uint8_t*)W->w_tc + (size_t)T0 * (K / 256) * qb_repacked_bytes_tc(128, 256);
                        seg.out = o + (size_t)T0 * 128;
                        seg.ldo = W->rows;
                        seg.rows = (int)(b - (uint64_t)T0 * 128);
                        if (wide)
                            CK(qb_qmv_tcw(&seg, 1, K, nn, s->xb, 0, (int)(a - (uint64_t)T0 * 128),
                                          (int)(b - (uint64_t)T0 * 128), s->work, s->st));
                        else
                            CK(qb_qmv_tc(&seg, 1, K, nn, s->xb, 0, (int)(a - (uint64_t)T0 * 128),
                                         (int)(b - (uint64_t)T0 * 128), s->work, s->st));
                    } else {
                        QbQSeg seg;
                        seg.w = (const uint8_t*)W->w + (size_t)t_lo * (K / qb_unit_cols(W->type)) * qb_unit_bytes(W->type);
                        seg.out = o + (size_t)t_lo * QB_TILE;
                        seg.ldo = W->rows;
                        seg.rows = (int)(b - (uint64_t)t_lo * QB_TILE);
                        CK(qb_qmv(W->type, &seg, 1, K, nn, s->xb, 0, (int)(a - (uint64_t)t_lo * QB_TILE),
                                  (int)(b - (uint64_t)t_lo * QB_TILE), s->work, s->st));
                    }
                    CK(cudaMemcpy2DAsync(outs[i] + (size_t)t0 * ldos[i] + a, ldos[i] * 4, o + a, (size_t)W->rows * 4,
                                         (size_t)(b - a) * 4, nn, cudaMemcpyDeviceToHost, s->st));
                }
                o += (size_t)nn * W->rows;
            }
            // the staging buffers are reused by the next chunk: its copies must have left
            CK(cudaStreamSynchronize(s->st));
        }
    }
    return 0;
}

int gemv_host(const gguf_tensor_info_t* W, const float* x, uint64_t ldx, int n, float* out, uint64_t ldo, uint64_t r0,
              uint64_t r1) {
    return gemv_multi_host(&W, 1, x, ldx, n, &out, &ldo, r0, r1);
}

int op_host(int which, float* out, const float* x, const float* w, uint64_t n, float eps) {
    std::lock_guard<std::mutex> lk(g_mu);
    Scratch* s = nullptr;
    if (scratch_get(s, n, n, 0)) return -1;
    CK(cudaMemcpyAsync(s->x, x, n * 4, cudaMemcpyHostToDevice, s->st));
    float* wd = nullptr;
    if (w) {
        CK(cudaMemcpyAsync(s->out, w, n * 4, cudaMemcpyHostToDevice, s->st));
        wd = s->out;
    }
    switch (which) {
    case 0: CK(qb_op_rmsnorm(s->x, s->x, wd, (long long)n, eps, s->st)); break;
    case 1: CK(qb_op_l2norm(s->x, s->x, (long long)n, eps, s->st)); break;
    case 2: CK(qb_op_act(0, s->x, (long long)n, s->st)); break;
    case 3: CK(qb_op_act(1, s->x, (long long)n, s->st)); break;
    case 4: CK(qb_op_act(2, s->x, (long long)n, s->st)); break;
    case 5: CK(qb_op_softmax(s->x, (long long)n, s->st)); break;
    }
    CK(cudaMemcpyAsync(out, s->x, n * 4, cudaMemcpyDeviceToHost, s->st));
    CK(cudaStreamSynchronize(s->st));
    return 0;
}
}  // namespace

extern "C" void gemv_rows(const gguf_tensor_info_t* W, const float* x, float* out, uint64_t r0, uint64_t r1) {
    gemv_host(W, x, W ? W->ne[0] : 0, 1, out, W ? W->ne[1] : 0, r0, r1);
}
extern "C" void gemv(pool_t*, const gguf_tensor_info_t* W, const float* x, float* out) {
    gemv_host(W, x, W ? W->ne[0] : 0, 1, out, W ? W->ne[1] : 0, 0, W ? W->ne[1] : 0);
}
extern "C" void gemv_rows_batch(const gguf_tensor_info_t* W, const float* x, uint64_t ldx, int n, float* out, uint64_t ldo,
                                uint64_t r0, uint64_t r1) {
    gemv_host(W, x, ldx, n, out, ldo, r0, r1);
}
extern "C" void gemv_batch(pool_t*, const gguf_tensor_info_t* W, const float* x, uint64_t ldx, int n, float* out,
                           uint64_t ldo) {
    gemv_host(W, x, ldx, n, out, ldo, 0, W ? W->ne[1] : 0);
}
extern "C" void gemv_multi(pool_t*, const gguf_tensor_info_t* const* Ws, const float* x, float* const* outs, int n_mat) {
    if (!Ws || n_mat < 1 || n_mat > QB_GEMV_MULTI_MAX || !Ws[0]) {
        set_err(-1, "gemv_multi: bad arguments (n_mat %d, at most %d)", n_mat, QB_GEMV_MULTI_MAX);
        return;
    }
    uint64_t ldos[QB_GEMV_MULTI_MAX];
    uint64_t K = 0;
    for (int i = 0; i < n_mat; ++i) {
        ldos[i] = Ws[i] ? Ws[i]->ne[1] : 0;
        K = std::max<uint64_t>(K, Ws[i] ? Ws[i]->ne[0] : 0);
    }
    gemv_multi_host(Ws, n_mat, x, K, 1, outs, ldos, 0, ~0ull);
}
extern "C" void gemv_multi_batch(pool_t*, const gguf_tensor_info_t* const* Ws, const float* x, uint64_t ldx, int n,
                                 float* const* outs, const uint64_t* ldos, int n_mat) {
    gemv_multi_host(Ws, n_mat, x, ldx, n, outs, ldos, 0, ~0ull);
}
extern "C" void rmsnorm(float* out, const float* x, const float* weight, uint64_t n, float eps) {
    op_host(0, out, x, weight, n, eps);
}
extern "C" void l2norm(float* out, const float* x, uint64_t n, float eps) { op_host(1, out, x, nullptr, n, eps); }
extern "C" void silu_inplace(float* x, uint64_t n) { op_host(2, x, x, nullptr, n, 0.f); }
extern "C" void sigmoid_inplace(float* x, uint64_t n) { op_host(3, x, x, nullptr, n, 0.f); }
extern "C" void softplus_inplace(float* x, uint64_t n) { op_host(4, x, x, nullptr, n, 0.f); }
extern "C" void softmax_inplace(float* x, uint64_t n) {
    if (n) op_host(5, x, x, nullptr, n, 0.f);
}

extern "C" uint32_t model_sample_greedy(const float* logits, uint32_t vocab_size) {
    if (!logits || vocab_size == 0) return 0;
    std::lock_guard<std::mutex> lk(g_mu);
    Scratch* s = nullptr;
    if (scratch_get(s, vocab_size, 0, 0)) return 0;
    uint32_t r = 0;
    if (cudaMemcpyAsync(s->x, logits, (size_t)vocab_size * 4, cudaMemcpyHostToDevice, s->st) != cudaSuccess ||
        qb_argmax_reset(s->keys, 1, s->st) != cudaSuccess ||
        qb_argmax(s->x, vocab_size, (int)vocab_size, 1, s->keys, s->st) != cudaSuccess ||
        qb_argmax_to_u32(s->keys, 1, s->am, s->st) != cudaSuccess ||
        cudaMemcpyAsync(&r, s->am, 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess ||
        cudaStreamSynchronize(s->st) != cudaSuccess) {
        set_err(-1, "model_sample_greedy: CUDA failure");
        return 0;
    }
    return r;
}

// ------------------------------ sampling ------------------------------------
// sampler_* keep the names, fields and behaviour of include/sampler.h /
// src/sampler.c; the draw itself runs on the device (qb_sample.cu).

namespace {
// device sampler state from the host sampler and the token history (its last
// QB_SAMP_HIST tokens land at their ring positions)
QbSampDev samp_state(const sampler_t* s, const uint32_t* tokens, size_t n_tokens) {
    QbSampDev h{};
    h.temp = s->temp;
    h.top_p = s->top_p;
    h.top_k = s->top_k;
    h.repeat_penalty = s->repeat_penalty;
    h.repeat_last_n = s->repeat_last_n;
    h.rng = s->rng_state;
    h.n_hist = tokens ? (uint32_t)n_tokens : 0u;
    const size_t m = h.n_hist < QB_SAMP_HIST ? h.n_hist : QB_SAMP_HIST;
    for (size_t i = h.n_hist - m; i < h.n_hist; ++i) h.hist[i % QB_SAMP_HIST] = tokens[i];
    return h;
}

int samp_alloc(QbSampDev*& sd, unsigned long long*& cand, unsigned long long*& keys, uint32_t*& am, int V) {
    if (sd) return 0;
    CK(cudaMalloc(&sd, sizeof(QbSampDev)));
    CK(cudaMalloc(&cand, (size_t)qb_sample_lists(V) * 256 * sizeof(unsigned long long)));
    CK(cudaMalloc(&keys, 2 * sizeof(unsigned long long)));
    CK(cudaMalloc(&am, 2 * sizeof(uint32_t)));
    return 0;
}
struct HostSamp {
    QbSampDev* sd = nullptr;
    unsigned long long *cand = nullptr, *keys = nullptr;
    uint32_t* am = nullptr;
    int V = 0;
};
std::unordered_map<int, HostSamp> g_hsamp;   // per device, for sampler_sample
}  // namespace

extern "C" sampler_t* sampler_init(float temp, float top_p, uint32_t top_k, float repeat_penalty, uint64_t seed) {
    sampler_t* s = (sampler_t*)calloc(1, sizeof(sampler_t));
    if (!s) return nullptr;
    s->temp = temp;
    s->top_p = top_p;
    s->top_k = top_k == 0 ? 40 : top_k;
    s->repeat_penalty = repeat_penalty <= 0.0f ? 1.0f : repeat_penalty;
    s->repeat_last_n = 64;
    s->rng_state = seed == 0 ? 0x123456789abcdefULL : seed;
    return s;
}

extern "C" void sampler_free(sampler_t* s) { free(s); }

// Host logits, as the reference: they are penalised in place (the same float
// operations, done on the device and copied back) and s->rng_state advances.
extern "C" uint32_t sampler_sample(sampler_t* s, float* logits, uint32_t vocab_size, const uint32_t* tokens,
                                   size_t n_tokens) {
    if (!s || !logits || vocab_size == 0) return 0;
    std::lock_guard<std::mutex> lk(g_mu);
    Scratch* sc = nullptr;
    if (scratch_get(sc, vocab_size, 1, 0)) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { set_err(-2, "sampler_sample: no device"); return 0; }
    HostSamp& hs = g_hsamp[dev];
    if (hs.sd && hs.V < (int)vocab_size) {   // the candidate lists grow with the vocabulary
        cudaFree(hs.sd); cudaFree(hs.cand); cudaFree(hs.keys); cudaFree(hs.am);
        hs = HostSamp();
    }
    if (samp_alloc(hs.sd, hs.cand, hs.keys, hs.am, (int)vocab_size)) return 0;
    hs.V = std::max(hs.V, (int)vocab_size);
    const QbSampDev h = samp_state(s, tokens, n_tokens);
    const bool penal = s->repeat_penalty != 1.0f && tokens && n_tokens > 0;
    QbSampDev out;
    if (cudaMemcpyAsync(sc->x, logits, (size_t)vocab_size * 4, cudaMemcpyHostToDevice, sc->st) != cudaSuccess ||
        cudaMemcpyAsync(hs.sd, &h, sizeof h, cudaMemcpyHostToDevice, sc->st) != cudaSuccess ||
        qb_sample(sc->x, (int)vocab_size, hs.sd, hs.cand, hs.keys, hs.am, sc->st) != cudaSuccess ||
        cudaMemcpyAsync(&out, hs.sd, sizeof out, cudaMemcpyDeviceToHost, sc->st) != cudaSuccess ||
        (penal && cudaMemcpyAsync(logits, sc->x, (size_t)vocab_size * 4, cudaMemcpyDeviceToHost, sc->st) != cudaSuccess) ||
        cudaStreamSynchronize(sc->st) != cudaSuccess) {
        set_err(-2, "sampler_sample: CUDA failure");
        return 0;
    }
    s->rng_state = out.rng;
    return out.token;
}

// src/main.c:232-248 with a sampler: token 0 = sample(m->logits), then
// n_predict - 1 steps of forward + sample, all on the device.  tokens /
// n_tokens: the history the repetition penalty sees (prompt and anything
// generated before); the new tokens extend it.
extern "C" int qb_sample_generate(qwen_model_t* m, sampler_t* s, uint32_t n_predict, const uint32_t* tokens,
                                  size_t n_tokens, uint32_t* out_tokens) {
    Engine* e = E_(m);
    if (!e || !s || !out_tokens || m->pos == 0) { set_err(-1, "qb_sample_generate: bad arguments"); return -1; }
    if (n_predict == 0) return 0;
    CK(cudaSetDevice(e->dev));
    if (ensure_out_buffers(*e, n_predict + 1, 1, 1)) return -1;
    if (samp_alloc(e->samp, e->samp_cand, e->samp_keys, e->samp_am, e->V)) return -1;
    if (!e->g_sample && capture(*e, &e->g_sample, record_sample, 0)) return -1;
    const QbSampDev h = samp_state(s, tokens, n_tokens);
    QbCtrl hc;
    CK(cudaMemcpyAsync(&hc, e->ctrl, sizeof hc, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    hc.fwd_pos = m->pos;
    hc.greedy_n = 0;
    hc.cap_out = e->cap_out;
    CK(cudaMemcpyAsync(e->ctrl, &hc, sizeof hc, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->samp, &h, sizeof h, cudaMemcpyHostToDevice, e->st));
    // the logits the caller holds (the last forward's, possibly edited) are the first draw's
    CK(cudaMemcpyAsync(e->logits, m->logits, (size_t)e->V * 4, cudaMemcpyHostToDevice, e->st));
    CK(qb_sample(e->logits, e->V, e->samp, e->samp_cand, e->samp_keys, e->samp_am, e->st));
    CK(qb_launch(sample_step_kernel, dim3(1), dim3(1), 0, e->st, e->ctrl, (const QbSampDev*)e->samp, e->d_out_tok, 0));
    uint32_t steps = n_predict - 1;
    if (m->pos + steps > (uint32_t)e->n_ctx) steps = (uint32_t)e->n_ctx - m->pos;
    CK(cudaEventRecord(e->ev0, e->st));
    for (uint32_t i = 0; i < steps; ++i) CK(cudaGraphLaunch(e->g_sample, e->st));
    CK(cudaEventRecord(e->ev1, e->st));
    CK(cudaEventSynchronize(e->ev1));
    cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
    const uint32_t n = steps + 1;
    QbSampDev out;
    CK(cudaMemcpyAsync(out_tokens, e->d_out_tok, (size_t)n * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaMemcpyAsync(&out, e->samp, sizeof out, cudaMemcpyDeviceToHost, e->st));
    // the logits the reference leaves: the last forward's, penalised by the last draw
    CK(cudaMemcpyAsync(m->logits, e->logits, (size_t)e->V * 4, cudaMemcpyDeviceToHost, e->st));
    if (dev_sync(*e)) return -1;
    s->rng_state = out.rng;
    m->pos += steps;
    return (int)n;
}

// ---------------------- allocation-free greedy argmax -------------------------
// For callers that must not allocate device memory at call time: code that
// owns every byte of the GPU through its own arena or pool, or runs where a
// cudaMalloc would synchronise the device or may fail under memory pressure.
// Same kernels as model_sample_greedy, but the per-row (value, index) keys
// live in this fixed file-scope array instead of library-allocated scratch.
static __device__ __align__(256) unsigned long long g_noalloc_keys[QB_ARGMAX_NOALLOC_MAX_ROWS];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned long long* g_noalloc_keys_ptr[kNoAllocMaxDevices] = {};   // per device, set on first use
}   // namespace

extern "C" int qb_argmax_rows_noalloc(const float* logits, int64_t ld, uint32_t n, uint32_t rows,
                                      uint32_t* out, void* stream) {
    if (!logits || !out || n == 0 || rows == 0) {
        set_err(-1, "qb_argmax_rows_noalloc: null pointer or empty size (n %u, rows %u)", n, rows);
        return -1;
    }
    if (rows > QB_ARGMAX_NOALLOC_MAX_ROWS) {
        set_err(-1, "qb_argmax_rows_noalloc: rows %u exceeds the static scratch maximum of %d", rows,
                QB_ARGMAX_NOALLOC_MAX_ROWS);
        return -1;
    }
    if (n > 0x7FFFFFFFu || ld < (int64_t)n) {
        set_err(-1, "qb_argmax_rows_noalloc: n %u must be < 2^31 and ld %lld >= n", n, (long long)ld);
        return -1;
    }
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        set_err(-1, "qb_argmax_rows_noalloc: device ordinal %d >= %d", dev, kNoAllocMaxDevices);
        return -1;
    }
    unsigned long long* keys = nullptr;
    {
        // set-up, once per device with that device current
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_keys_ptr[dev]) {
            void* p = nullptr;
            CK(cudaGetSymbolAddress(&p, g_noalloc_keys));
            g_noalloc_keys_ptr[dev] = static_cast<unsigned long long*>(p);
        }
        keys = g_noalloc_keys_ptr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CK(qb_argmax_reset(keys, (int)rows, st));   // the keys of the previous call are stale
    CK(qb_argmax(logits, ld, (int)n, (int)rows, keys, st));
    CK(qb_argmax_to_u32(keys, (int)rows, out, st));
    return 0;
}
