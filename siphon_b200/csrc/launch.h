// Host-side launch helpers shared by the kernels' translation units and the
// C ABI (abi.cu). Return 0 on success, negative on a launch problem.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sicu {

constexpr int MAX_MATS = 64;

struct GemvLaunch {
    const void *w;        // weight blocks (device), single-matrix launches
    const void *xq;       // pair-format activation (device) or null
    const float *xf;      // f32 activation (device) for the fused quantizer, or null
    float *y;             // [n_out] (device), single-matrix launches
    int64_t n_out;
    int n_in;
    // matrices of the launch (same format, same n_in, one activation):
    // filled from w / y / n_out when nmat == 1
    int nmat;
    const void *wm[MAX_MATS];
    float *ym[MAX_MATS];
    int64_t n_outm[MAX_MATS];
    int num_sms;
    int smem_limit;       // opt-in dynamic shared memory per block
    int smem_per_sm;      // shared memory per multiprocessor
    int smem_reserved;    // shared memory the runtime reserves per block
    int overlap;          // programmatic dependent launch: weights may stream before
                          // earlier work in the stream completes
    int device;
    int *status;          // device status word
};

// quantized formats (K and classic); fails with -3 for other types
int launch_gemv(uint32_t wtype, const GemvLaunch &L, cudaStream_t st);
// F16 weights (pair activation: f16 row, or f32 converted in the kernel)
int launch_gemv_f16(const GemvLaunch &L, cudaStream_t st);

// activation conversion of m rows of n floats into the pair format
int launch_quantize(uint32_t pair, const float *x, void *y, int64_t n, int64_t m, cudaStream_t st);

// prefill matrix product on the tensor cores: y[t][r] for m tokens (Q8_K rows)
struct PrefillLaunch {
    const void *w;        // weight blocks (device)
    int64_t n_in, n_out;
    const void *xq;       // m rows of Q8_K blocks (device)
    int64_t m;
    float *y;             // [m][n_out] (device)
    void *ws;             // prefill_workspace_bytes(wtype, n_in, n_out, m) bytes, 256-byte aligned
    int device;
    int *status;
};
bool prefill_supported(uint32_t wtype);
size_t prefill_workspace_bytes(uint32_t wtype, int64_t n_in, int64_t n_out, int64_t m);
// -3: no tensor-core kernel for the type; -4: tensor map encoding failed; -2: launch
int launch_prefill(uint32_t wtype, const PrefillLaunch &L, cudaStream_t st);

// dequantise rows (row_to_f32): rows[i] of w into out[i * n_in]
int launch_dequant(uint32_t wtype, const void *w, int64_t n_in, const int64_t *rows_dev, int64_t nrows,
                   float *out, cudaStream_t st);

}  // namespace sicu
