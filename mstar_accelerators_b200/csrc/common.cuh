// Shared host/device helpers of libmstar_b200 (sm_100a).
//
// Device layouts (B200 layout of the canonical ggml blocks; same bytes per
// block: 34 for Q8_0, 18 for Q4_0):
//
//  Weights are the B operand of mma.m16n8k32 (K x N, "col"): lane (g, t) of a
//  warp holds b0 = W[row g][k 4t..4t+3] and b1 = W[row g][k 16+4t..16+4t+3].
//  Rows are grouped by 8 ("row group" G = row / 8, padded with zero rows).
//   Q8_0 quants: wq[G][pair p][lane][16 B]: {block 2p: b0, b1; block 2p+1: b0, b1}
//   Q4_0 quants: wq[G][quad q][lane][16 B]: {block 4q+j: qs[4t..4t+3]}, j = 0..3;
//                the low nibbles of those 4 bytes are b0 (elements 4t..4t+3)
//                and the high nibbles b1 (elements 16+4t..), value = nibble - 8.
//   scales:      ws[G][block][8 rows] fp16 (row fastest); lane (g, t) reads the
//                half2 of rows 2t, 2t+1 — the two output columns it owns.
//  One 16-byte load per lane per warp-step moves 512 contiguous bytes.
//
//  Activations are the A operand (M x K, "row"): the quantizer writes them
//  directly in fragment order, xf[block][mtile][lane][16 B] = {a0, a1, a2, a3}
//  with a0 = X[g][4t..], a1 = X[g+8][4t..], a2 = X[g][16+4t..],
//  a3 = X[g+8][16+4t..] for the 16 tokens of the tile, and the fp32 value of
//  each stored fp16 scale in xs[block][token].
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace mb {

constexpr int QK = 32;
constexpr int Q8_BYTES = 34;
constexpr int Q4_BYTES = 18;

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void require(bool ok, const char *what) {
    if (!ok) throw Error(what);
}

inline void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline void message(char *p, size_t n, const char *e) {
    if (p && n) std::snprintf(p, n, "%s", e);
}

struct Range {
    const void *data;
    uint64_t bytes;
};

inline bool disjoint(Range a, Range b) {
    if (!a.bytes || !b.bytes) return true;
    const uintptr_t x = uintptr_t(a.data), y = uintptr_t(b.data);
    return x + a.bytes <= y || y + b.bytes <= x;
}

// Extent/alignment check of a borrowed range (decoder.cpp:29-32 semantics).
inline void check_range(Range r, uint64_t bytes, size_t alignment, const char *what) {
    if (!(r.data && r.bytes == bytes && uintptr_t(r.data) % alignment == 0 &&
          uintptr_t(r.data) <= UINTPTR_MAX - bytes))
        throw Error(std::string("invalid borrowed storage extent/alignment: ") + what);
}

// A borrowed pointer must be device-accessible memory of the current device.
inline void check_device(const void *p, const char *what) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        throw Error(std::string("not a CUDA pointer: ") + what);
    }
    int dev = -1;
    cudaGetDevice(&dev);
    if (!((a.type == cudaMemoryTypeDevice && a.device == dev) || a.type == cudaMemoryTypeManaged))
        throw Error(std::string("not device memory of the current device: ") + what);
}

inline cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Process-wide limits of the bounded device waits, in polls (0 = the built-in
// default). Set through mstar_b200_set_wait_limits; kernels launched afterwards
// use them (a decode-step handle reads them when it is created).
struct WaitLimits {
    long long tp_barrier = 0;    // k_tp_barrier: polls of ~100 ns
    long long grid_barrier = 0;  // persistent decode step: polls of ~64 ns
};
WaitLimits &wait_limits();

}  // namespace mb

// ---------------------------------------------------------------- device side
#ifdef __CUDACC__
namespace mb {

__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t word(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// D = A(16x32 s8, row) * B(32x8 s8, col), int32, C = 0.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0));
}

// D = A(16x32 s8, row) * B(32x8 u8, col), int32, C = 0 (Q4_0 nibbles as u8).
__device__ __forceinline__ void mma_s8u8(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0));
}

// Packed fp32 pairs (sm_100 f32x2 pipe): each lane is an IEEE RN operation,
// bit-identical to the scalar __fmul_rn / __fadd_rn.
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 r;
    asm("{.reg .b64 ra, rb, rc; mov.b64 ra, {%2,%3}; mov.b64 rb, {%4,%5}; mul.rn.f32x2 rc, ra, rb; "
        "mov.b64 {%0,%1}, rc;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 r;
    asm("{.reg .b64 ra, rb, rc; mov.b64 ra, {%2,%3}; mov.b64 rb, {%4,%5}; add.rn.f32x2 rc, ra, rb; "
        "mov.b64 {%0,%1}, rc;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
// Exact int -> float for |i| < 2^22 (every Q8_0/Q4_0 block dot is below
// 32*127*127 < 2^19): the integer is added to the bit pattern of 1.5*2^23,
// whose unit in the last place is 1, and the bias is subtracted again.
__device__ __forceinline__ float2 i2f2(int a, int b) {
    const float2 biased = make_float2(__int_as_float(a + 0x4B400000), __int_as_float(b + 0x4B400000));
    float2 r;
    asm("{.reg .b64 ra, rb, rc; mov.b64 ra, {%2,%3}; mov.b64 rb, {%4,%4}; sub.rn.f32x2 rc, ra, rb; "
        "mov.b64 {%0,%1}, rc;}"
        : "=f"(r.x), "=f"(r.y) : "f"(biased.x), "f"(biased.y), "f"(12582912.0f));
    return r;
}

// ---- bulk asynchronous copies (TMA, 1-D) tracked by an mbarrier -------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// One try_wait suspends the thread for up to a system-dependent time limit.
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Wait for phase `parity` of an mbarrier with an iteration limit; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t limit = 1u << 18) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---- 16-byte asynchronous global -> shared copies (cp.async, no TMA) ---------
// src_bytes 0 zero-fills the destination without reading the source.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Four 8x8 fp16 matrices from shared memory, transposed (ldmatrix .trans):
// thread 8 m + r gives the address of row r of matrix m.
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(row)));
}

// Q4_0 nibbles of 4 bytes -> (elements 4t..4t+3, elements 16+4t..) as unsigned
// nibbles; the -8 offset is applied after the dot as -8 * (sum of the block's
// activation quants), which keeps the integer result exact.
__device__ __forceinline__ void unpack_q4(uint32_t q, uint32_t &lo, uint32_t &hi) {
    lo = q & 0x0F0F0F0Fu;
    hi = (q >> 4) & 0x0F0F0F0Fu;
}

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor still runs;
// pdl_wait() blocks until the predecessor grid has completed and its memory is
// visible, pdl_trigger() lets this kernel's own dependent start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialization (the kernel must pdl_wait()
// before reading what earlier kernels wrote).
template <class... K, class... A>
inline void launch_pdl(void (*kernel)(K...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<K>(args)...);
}

// bits of a packed half2 (for 16-byte vector stores)
__device__ __forceinline__ uint32_t half2_bits(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, sizeof(u));
    return u;
}

// ggml stock GELU (ggml-cpu/vec.h:963-969, 1000-1013): x <= -10 gives 0,
// x >= 10 gives x, anything else the entry of ggml's fp16 table indexed by the
// fp16 bits of x. The table (gelu.cu) is built on the host exactly as the CPU
// backend builds its own at start-up (ggml-cpu.c:3889, with the host's tanhf),
// restricted to the entries -10 < x < 10 can reach (|h| <= 10): entry
// (bits & 0x7FFF) for +h, 0x4901 + (bits & 0x7FFF) for -h.
constexpr uint32_t GELU_HALF_ENTRIES = 0x4901u;                  // fp16 magnitudes 0 .. 10.0
constexpr int GELU_TABLE_ENTRIES = int(2 * GELU_HALF_ENTRIES);   // 37378 x 2 bytes
constexpr size_t GELU_TABLE_BYTES = (size_t(GELU_TABLE_ENTRIES) * 2 + 15) / 16 * 16;

__device__ __forceinline__ float gelu_ggml(float x, const uint16_t *table) {
    const uint32_t bits = __half_as_ushort(__float2half_rn(x));
    const uint32_t mag = min(bits & 0x7FFFu, GELU_HALF_ENTRIES - 1u);  // NaN and |x| >= 10 are decided below
    const float t = __half2float(__ushort_as_half(table[mag + ((bits & 0x8000u) ? GELU_HALF_ENTRIES : 0u)]));
    const float r = x <= -10.0f ? 0.0f : t;
    return x >= 10.0f || x != x ? x : r;
}

// ggml's GELU table on the current device (built and uploaded on first use,
// synchronises: call it outside stream capture).
const uint16_t *gelu_table();

// ggml_gelu_erf (ggml-cpu/vec.h:1024-1029).
__device__ __forceinline__ float gelu_erf(float x) {
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752440f))));
}

// Total order used by the fused argmax: NaN above everything, +0 == -0,
// and ties resolved toward the smaller index (decoder.cpp:686-696).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    uint32_t o;
    if (v != v) o = 0xFFFFFFFFu;
    else {
        if (v == 0.0f) v = 0.0f;
        const uint32_t b = __float_as_uint(v);
        o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    }
    return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - index);
}

}  // namespace mb
#endif
