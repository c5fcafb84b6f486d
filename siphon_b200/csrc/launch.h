// Host-side launch helpers shared by the kernels' translation units and the
// C ABI (abi.cu). Return 0 on success, negative on a launch problem.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sicu {

constexpr int MAX_MATS = 64;

// All-reduce group of a tensor-parallel decode, as the kernels see it. Every
// rank owns one peer-mapped allocation:
//   slot[2][n][len]  u64 tagged elements: (tag << 32) | f32 bits, double
//                    buffered by delivery parity
//   epoch[4]         u32, this rank only: [0] deliveries made, [2] CTA arrival
//                    counter, [3] broken (a wait timed out)
// Delivery k (1-based) of rank r stores element i as one 64-bit word with tag
// k into slot[(k - 1) & 1][r][i] of every rank; each rank reads
// slot[(k - 1) & 1][q][i] of its own memory for every q until the word
// carries tag k, so value and readiness arrive in one single-copy-atomic
// store. Rank q's delivery k + 2 (same buffer) cannot start before every rank
// finished reading delivery k: it follows q's delivery k + 1, which waited
// for every rank's part k + 1, which each rank sends only after its own
// delivery k completed.
constexpr int AR_MAX = 8;
struct ArDev {
    int n = 0, rank = 0;
    int64_t len = 0;                  // elements per partial
    uint64_t limit_ns = 0;            // bound of a consumption's wait
    uint64_t *slot[AR_MAX] = {};      // slot array of rank q (this rank's own at [rank])
    unsigned *epoch = nullptr;        // this rank's epoch words
};
// byte offsets inside one rank's allocation
inline int64_t ar_epoch_offset(int n, int64_t len) { return 2 * (int64_t)n * len * 8; }
inline int64_t ar_alloc_bytes(int n, int64_t len) { return ar_epoch_offset(n, len) + 16; }

// Activation step between two products of the reference's forward pass,
// applied by the product's quantizer to the f32 activation x (n_in floats)
// before it quantizes:
//   PRO_RMS_NORM  h = x (+ res: the residual add), a = h * rms_scale(h) * g,
//                 h also written to h_out when given (by the first cluster)
//   PRO_SWIGLU    a = silu(x) * up
//   PRO_MUL       a = x * up (SwiGLU's product when x already holds silu(gate),
//                 written by the gate product's silu epilogue)
constexpr int PRO_NONE = 0, PRO_RMS_NORM = 1, PRO_SWIGLU = 2, PRO_MUL = 3;
struct ProDev {
    int kind = PRO_NONE;
    float eps = 0.0f;
    const float *g = nullptr;      // norm weight [n_in]
    const float *res = nullptr;    // residual [n_in] or null
    float *h_out = nullptr;        // x + res [n_in] or null
    const float *up = nullptr;     // SwiGLU / MUL: up projection [n_in]
    double inv_n = 0.0;            // RMS norm: 1.0 / n_in
};

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
    ArDev ar;             // n > 0: row-split product, y = the group's sum of the partial outputs
    ProDev pro;           // step applied to xf before quantizing (quantized types)
    uint64_t epi_silu;    // bit i: matrix i's outputs are written as silu(y)
    const float *bias[MAX_MATS];   // matrix i's outputs get bias[i][row] added (null: none)
};

// quantized formats (K and classic); fails with -3 for other types
int launch_gemv(uint32_t wtype, const GemvLaunch &L, cudaStream_t st);
// F16 weights (pair activation: f16 row, or f32 converted in the kernel)
int launch_gemv_f16(const GemvLaunch &L, cudaStream_t st);

// n floats (a multiple of 4, 16-byte aligned) from the device view of
// page-locked host memory into device memory
int launch_host_copy(const float *src, float *dst, int64_t n, cudaStream_t st);

// activation conversion of m rows of n floats into the pair format
int launch_quantize(uint32_t pair, const float *x, void *y, int64_t n, int64_t m, cudaStream_t st);

// prefill matrix product on the tensor cores: y[t][r] for m tokens (Q8_K rows)
constexpr int PREFILL_MAXM = 4;            // matrices per grouped prefill launch
constexpr int PREFILL_PACKED_MIN_M = 32;   // blocks of more tokens than this read the prefill copies
struct PrefillLaunch {
    const void *w;        // weight blocks (device)
    int64_t n_in, n_out;
    const void *xq;       // m rows of Q8_K blocks (device), or null with xf set
    const float *xf;      // m rows of f32 (device, 16-byte aligned), quantized inside the launch
    int64_t m;
    float *y;             // [m][n_out] (device)
    void *ws;             // prefill_workspace_bytes(wtype, n_in, n_out, m, num_sms, pack != 0) bytes, 256-byte aligned
    int device;
    int num_sms;
    int *status;
    const void *pack;     // the prefill copy of w (prefill_pack_bytes), or null
    // more matrices that read the same activation (prefill copies required):
    // nmat > 1 lists every matrix of the group (entry 0 included) below
    int nmat = 1;
    const void *packm[PREFILL_MAXM];
    int64_t n_outm[PREFILL_MAXM];
    float *ym[PREFILL_MAXM];
};
// Q4_K, Q6_K: tensor-core kernels from the raw blocks (converters) and from
// the prefill copies
bool prefill_supported(uint32_t wtype);
// Q2_K ... Q6_K: a prefill copy and the kernels that read it (m > 32 tokens);
// Q2_K, Q3_K and Q5_K have no converter kernel, so without a copy of their own
// a product first makes one in the workspace
bool prefill_pack_supported(uint32_t wtype);
// Q4_0, Q5_0, Q8_0: int8 tensor-core kernel from the prefill copy (m > 32,
// n_in >= 128), bit-identical with the per-token matvec
bool is_classic(uint32_t wtype);
// formats whose copies several products on one activation can share a launch with
bool prefill_groupable(uint32_t wtype);
size_t prefill_workspace_bytes(uint32_t wtype, int64_t n_in, int64_t n_out, int64_t m, int num_sms, bool packed);
// a group of nmat matrices read from their prefill copies (m > 32)
size_t prefill_group_workspace_bytes(uint32_t wtype, int64_t n_in, int nmat, const int64_t *n_out, int64_t m,
                                     int num_sms);
// bytes of the prefill copy of an n_out x n_in matrix (0: no tensor-core kernel for the type)
size_t prefill_pack_bytes(uint32_t wtype, int64_t n_in, int64_t n_out);
// writes the prefill copy of the weight blocks w into pack; -3: unsupported type
int launch_prefill_pack(uint32_t wtype, const void *w, int64_t n_in, int64_t n_out, void *pack, cudaStream_t st);
// -3: no tensor-core kernel for the type (or, for a type without converters,
// no copy or m <= 32); -4: tensor map encoding failed; -2: launch
int launch_prefill(uint32_t wtype, const PrefillLaunch &L, cudaStream_t st);

// batch decode matvec on the tensor cores: y[i][t][r] = (W_i x_t)[r] for
// t < m <= 8 activation rows, every weight block read once for all of them;
// bit-identical with the per-token matvec (Q4_K and Q6_K)
constexpr int BATCH_MAX = 8;
struct BatchLaunch {
    int nmat;                     // 1..16 matrices of one type and row length
    const void *w[16];
    float *y[16];                 // [m][n_out[i]] each (device)
    int64_t n_out[16];
    int64_t n_in;
    const float *xf;              // m f32 rows (device), or null with xq set
    const void *xq;               // m Q8_K rows (device)
    int m;
    void *ws;                     // batch_workspace_bytes(n_in) bytes, 16-byte aligned
    int num_sms, smem_per_sm, smem_reserved;
    int overlap;                  // programmatic dependent launch of the prep kernel
    int device;
    int *status;
};
bool batch_supported(uint32_t wtype);
size_t batch_workspace_bytes(int64_t n_in);
// -1: bad launch (matrix or row count); -3: type without a batch kernel; -2: launch
int launch_batch(uint32_t wtype, const BatchLaunch &L, cudaStream_t st);

// the activation steps on their own, m rows of n floats (f32 out): RMS norm
// (res, h_out per row, or null) and SwiGLU (n * m a multiple of 4)
int launch_rms_norm(const float *x, const float *res, float *h_out, const float *g, int64_t n, int64_t m,
                    float eps, float *y, cudaStream_t st);
int launch_swiglu(const float *x, const float *up, int64_t n, int64_t m, float *y, cudaStream_t st);
// y = x * up, n floats
int launch_mul(const float *x, const float *up, int64_t n, float *y, cudaStream_t st);
// y = silu(y), n floats in place (F16 products with a silu epilogue)
int launch_silu_inplace(float *y, int64_t n, cudaStream_t st);
// y += b, n floats in place (F16 products with a bias epilogue)
int launch_add_inplace(float *y, const float *b, int64_t n, cudaStream_t st);
// y_r += b for m rows of n floats (the Q/K/V bias adds of a prompt)
int launch_add_rows(float *y, const float *b, int64_t n, int64_t m, cudaStream_t st);

// the reference's attention softmax over m rows of n floats (row maximum
// taken here); in place allowed
int launch_softmax(const float *x, float *y, int64_t n, int64_t m, cudaStream_t st);
// attention of one position over the f16 caches of one layer (one CTA per
// query head), RoPE in place, and the K/V store of one position
int launch_attention(const float *q, const void *kc, const void *vc, int n_head, int n_head_kv, int hd, int n_ctx,
                     int pos, float ks, float *out, cudaStream_t st);
int launch_rope(float *x, int n_heads, int hd, int n_rot, const float *cs, const float *sn, int neox, cudaStream_t st);
int launch_kv_store(const float *k, const float *v, void *kc, void *vc, int n_head_kv, int hd, int n_ctx, int pos,
                    cudaStream_t st);
// the three in one launch (overlap: unused; the launch always waits for the
// previous kernel to finish)
// a prompt's m consecutive positions pos0..pos0+m-1: RoPE, the K/V store and
// every (head, token)'s attention over its prefix (two launches)
int launch_attention_prompt(const float *q, const float *k, const float *v, void *kc, void *vc, const float *cs,
                            const float *sn, int n_head, int n_head_kv, int hd, int n_rot, int neox, int n_ctx, int pos0,
                            int m, float ks, float *out, cudaStream_t st);
int launch_attention_step(const float *q, const float *k, const float *v, void *kc, void *vc, const float *cs,
                          const float *sn, int n_head, int n_head_kv, int hd, int n_rot, int neox, int n_ctx, int pos,
                          float ks, float *out, int overlap, cudaStream_t st);

// all-reduce of src[len] into dst[len] over the group (one delivery)
int launch_allreduce(const ArDev &a, const float *src, float *dst, int *status, int num_sms, cudaStream_t st);

// dequantise rows (row_to_f32): rows[i] of w into out[i * n_in]; row ids
// outside [0, n_rows) give a NaN row and STATUS_BAD_ROW in *status
int launch_dequant(uint32_t wtype, const void *w, int64_t n_in, const int64_t *rows_dev, int64_t nrows,
                   float *out, cudaStream_t st, int64_t n_rows = INT64_MAX, int *status = nullptr);
// greedy choice (first maximum) of m rows of n floats into out[m]
int launch_argmax(const float *x, int64_t n, int64_t m, int64_t *out, cudaStream_t st);

}  // namespace sicu
