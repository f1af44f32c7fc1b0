// Shared device helpers and launch-parameter structs for the sm_100a kernels.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#define QB_TILE 16          // rows per tensor-core tile (m16n8k16 M dimension)
#define QB_MAX_TOK 8        // verify / prefill width handled by one GEMV launch
#define QB_WIDE 32          // rows of one multi-sequence forward (QB_MAX_TOK-row chunks per GEMV launch)
#define QB_MAX_SEQ 8        // sequences of one multi-sequence forward
#define QB_MAX_SEG 4        // matrices fused into one GEMV launch (shared input)

// ggml type ids, identical to the GGUF numbering (reference include/gguf.h:40-64)
enum QbType : int { QB_F32 = 0, QB_Q8_0 = 8, QB_Q4_K = 12, QB_Q5_K = 13, QB_Q6_K = 14, QB_IQ4_XS = 23 };

// Bytes of one repacked (16-row tile x 256-column super-block) unit.  Q8_0 uses
// a (16-row tile x 32-column block) unit.  The K-quant and Q8_0 layouts hold
// exactly the bytes of the 16 source rows (the repack only reorders them);
// IQ4_XS keeps 2 more bytes per row (138 instead of 136): its 6-bit sub-block
// scales are stored expanded, as the int8 differences the GEMV applies.
__host__ __device__ constexpr int qb_unit_bytes(int type) {
    return type == QB_IQ4_XS ? 16 * 138
         : type == QB_Q6_K   ? 16 * 210
         : type == QB_Q4_K   ? 16 * 144
         : type == QB_Q5_K   ? 16 * 176
         : type == QB_Q8_0   ? 16 * 34
         : 0;
}
__host__ __device__ constexpr int qb_unit_cols(int type) { return type == QB_Q8_0 ? 32 : 256; }

struct QSeg {
    const uint8_t* w;     // repacked weights of this matrix
    float* out;           // out[t * ldo + row]
    long long ldo;
    int rows;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// D = A(16x16, f16, row) * B(16x8, f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A(16x16, f16, row) * B(16x8, f16, col), fp32 (zero accumulator input).
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// D = A(16x32, s8, row) * B(32x8, s8, col) + C, exact int32 accumulate.
__device__ __forceinline__ void mma_16832_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float h2f_bits(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)(h16 & 0xFFFFu)));
}

// exact small-integer -> float for 0 <= v < 2^22 without I2F: (2^23 + v) - 2^23
__device__ __forceinline__ float small_u2f(uint32_t v) {
    return __int_as_float(0x4B000000u | v) - 8388608.0f;
}

// ---- waits on other ranks ----
// A wait on a peer gives up after kPeerWaitNs of wall-clock time (%globaltimer),
// or at once when the error word already records a failed wait, so that a
// rank that stopped taking part costs one bound, not one per exchange.
constexpr unsigned long long kPeerWaitNs = 2000000000ull;
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// true: stop waiting (the error word is set, to code when this wait ran out)
__device__ __forceinline__ bool peer_wait_over(uint32_t it, unsigned long long t0, unsigned* err, unsigned code) {
    if (it & 63u) return false;
    if (*(volatile unsigned*)err) return true;
    if (global_ns() - t0 > kPeerWaitNs) {
        atomicExch(err, code);
        return true;
    }
    return false;
}

// ---- programmatic dependent launch (PDL) ----
// Every kernel calls pdl_wait() before it touches data written by (or read
// by) the kernel before it on the stream, and pdl_trigger() once it no longer
// needs to hold back the next kernel's launch.  Without the launch attribute
// both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

#include <utility>
template <typename... KArgs, typename... Args>
inline cudaError_t qb_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---- shared-memory / mbarrier / bulk-copy helpers (sm_90+ PTX) ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
// Plain loads (not asm): ordered after an mbarrier wait by its memory clobber,
// otherwise free for the scheduler to interleave.
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ int lds_s8(const uint8_t* p) { return *reinterpret_cast<const int8_t*>(p); }

// 4-byte global -> shared copy completed by cp_async_wait_all (this thread's copies)
__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
// device-scope atomic add with acquire-release semantics; returns the old value
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// bounded wait on phase parity; returns false when the bound was hit
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_iter = (1u << 22)) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t it = 0; it < max_iter; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
// bounded wait that lets the hardware suspend the thread up to hint_ns per try
// instead of spinning; returns false when the bound was hit
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns,
                                                uint32_t max_iter = (1u << 16)) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t it = 0; it < max_iter; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(hint_ns)
            : "memory");
        if (ok) return true;
    }
    return false;
}
// the same two operations on shared-memory addresses already in the shared window
__device__ __forceinline__ void mbar_expect_tx_s(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s_s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// 1-D bulk copy global -> shared, completion counted on the mbarrier
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
