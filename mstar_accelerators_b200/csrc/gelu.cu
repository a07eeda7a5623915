// ggml's fp16 GELU table (see gelu_ggml in common.cuh).
//
// ggml evaluates its stock GELU through a 65536-entry fp16 table that the CPU
// backend fills at start-up with the host's tanhf (ggml_gelu_f32,
// ggml-cpu/vec.h:1000-1004; table at ggml-cpu.c:3889). The kernels look the
// same entries up: this file computes them on the host in ggml's operation
// order and keeps the 37378 entries that inputs -10 < x < 10 can reach on each
// device (73 KB; the GEMM epilogue copies them to shared memory).
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace mb {

// ggml_gelu_f32 stored as fp16, in the same operation order, single precision.
static uint16_t host_table_entry(uint16_t bits) {
    __half_raw raw;
    raw.x = bits;
    const float x = __half2float(__half(raw));
    const float sqrt_2_over_pi = 0.79788456080286535587989211986876f, coef_a = 0.044715f;
    const float inner = sqrt_2_over_pi * x * (1.0f + coef_a * x * x);
    const float g = 0.5f * x * (1.0f + tanhf(inner));
    const __half_raw out = __half(__float2half_rn(g));
    return out.x;
}

const uint16_t *gelu_table() {
    static std::mutex lock;
    static std::vector<uint16_t *> per_device;
    std::lock_guard<std::mutex> guard(lock);
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "current device");
    if (int(per_device.size()) <= dev) per_device.resize(dev + 1, nullptr);
    if (per_device[dev]) return per_device[dev];
    std::vector<uint16_t> host(GELU_TABLE_BYTES / 2, 0);
    for (uint32_t m = 0; m < GELU_HALF_ENTRIES; ++m) {
        host[m] = host_table_entry(uint16_t(m));
        host[GELU_HALF_ENTRIES + m] = host_table_entry(uint16_t(0x8000u | m));
    }
    uint16_t *table = nullptr;
    cuda_check(cudaMalloc(&table, GELU_TABLE_BYTES), "GELU table");
    const cudaError_t e = cudaMemcpy(table, host.data(), GELU_TABLE_BYTES, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(table);
        cuda_check(e, "GELU table upload");
    }
    per_device[dev] = table;  // kept for the life of the process, like the library's kernels
    return table;
}

}  // namespace mb
