#pragma once
// The prepared block-quantized linear behind a mstar_b200_linear_* handle
// (abi.cu), shared with the persistent decode-step kernel (step.cu), which
// reads the prepared weight fragments of the handles it is built from.
#include <atomic>

#include <cuda.h>

#include "common.cuh"

namespace mb {

struct Linear {
    int q4 = 0;
    int64_t rows = 0, width = 0, nb = 0, nb_pad = 0, groups = 0;
    uint4 *wq = nullptr;
    __half *ws = nullptr;
    float *bias = nullptr;
    // per-handle device state shared by every call: calls on one handle must
    // be ordered on the device (one stream, or explicit events).
    uint32_t *xf = nullptr;  // activation fragments of one 32-query chunk
    float *xs = nullptr;
    int *xsum = nullptr;
    int *status = nullptr;
    unsigned long long *keys = nullptr;
    unsigned int *done = nullptr;
    int wpg_override = 0;  // > 0 forces the split-K fold (tests)
    const uint16_t *gelu = nullptr;  // ggml GELU table of the handle's device
    bool gemv_ok = true;   // the decode GEMV's shared-memory tile fits this width (K <= 4096)
    // tcgen05 GEMM state for calls with more than GEMM_MIN_QUERIES rows
    __half *w16 = nullptr;        // fp16(q * d) weights [rows][width]
    __half *x16 = nullptr;        // fp16 dequantized activations [gemm_rows][width]
    int64_t gemm_rows = 0;
    CUtensorMap wmap{};       // 256-row boxes (single-CTA GEMM)
    CUtensorMap wmap_pair{};  // 128-row boxes (CTA-pair GEMM)
    // vocab readout tile layout (readout.cu), built by prepare_readout
    uint8_t *wt = nullptr;
    int64_t tiles = 0;
    int *ro_flags = nullptr;  // status bits of the readout in flight
    std::atomic_flag busy = ATOMIC_FLAG_INIT;
    uint64_t weight_bytes() const { return uint64_t(groups) * 8 * nb_pad * (q4 ? 18 : 34); }
    ~Linear() {
        for (void *p : {(void *)wq, (void *)ws, (void *)bias, (void *)xf, (void *)xs, (void *)xsum, (void *)status, (void *)keys,
                        (void *)done, (void *)w16, (void *)x16, (void *)wt, (void *)ro_flags})
            if (p) cudaFree(p);
    }
};

struct Busy {
    std::atomic_flag &flag;
    explicit Busy(std::atomic_flag &f) : flag(f) {
        require(!flag.test_and_set(std::memory_order_acquire), "linear handle is busy");
    }
    ~Busy() { flag.clear(std::memory_order_release); }
};

}  // namespace mb
