/* siphon: CUDA backend for the reference's backend vtable (include/siphon/
 * tensor.h:43-55), over libsiphon_cuda (include/siphon_cuda.h).
 *
 * The host side a maintainer adds to the reference as src/backend_cuda.c:
 * the `gemv` slot runs the matvec on the GPU through sicu_gemv_host (host x
 * in, host y out, synchronous, results bit-identical to cpu_gemv's scalar
 * dots); weight blocks are uploaded once, on first use, straight from the
 * GGUF mmap. The `row_to_f32` slot (the embedding lookup, src/engine.c:
 * 300-304) dequantizes the row on the device (sicu_row_to_f32, the
 * reference's si_dequant_row semantics) and copies it back.
 *
 * Built against the reference's headers; the reference's si_set_err is
 * resolved from the process it is loaded into. */
#include "siphon/tensor.h"
#include "siphon_cuda.h"

#define SICU_BE_MAX_TENSORS 8192

typedef struct {
    const void *host;   /* GGUF mmap pointer of the tensor */
    void *dev;          /* device copy */
} dev_entry;

static dev_entry g_tab[SICU_BE_MAX_TENSORS];
static int g_ntab;
static int g_last;

static void *device_copy(const si_tensor *w) {
    if (g_ntab && g_tab[g_last].host == w->data) return g_tab[g_last].dev;
    for (int i = 0; i < g_ntab; i++) {
        if (g_tab[i].host == w->data) {
            g_last = i;
            return g_tab[i].dev;
        }
    }
    if (g_ntab == SICU_BE_MAX_TENSORS) {
        si_set_err("cuda backend: more than %d weight tensors", SICU_BE_MAX_TENSORS);
        return NULL;
    }
    void *dev = NULL;
    if (sicu_upload(w->data, (size_t)w->n_bytes, &dev) != SICU_OK) {
        char msg[256];
        sicu_last_error(msg, sizeof msg);
        si_set_err("cuda backend: upload: %s", msg);
        return NULL;
    }
    g_tab[g_ntab].host = w->data;
    g_tab[g_ntab].dev = dev;
    g_last = g_ntab++;
    return dev;
}

static void cuda_gemv(si_backend *be, const si_tensor *w, const float *x, float *y,
                      int64_t n_out, si_tp *tp) {
    (void)be;
    (void)tp;
    void *dw = device_copy(w);
    if (!dw) return;
    if (sicu_gemv_host(w->type, dw, (int64_t)w->ne[0], n_out, x, y, NULL) != SICU_OK) {
        char msg[256];
        sicu_last_error(msg, sizeof msg);
        si_set_err("cuda gemv: %s", msg);
    }
}

static float *g_row;          /* device buffer of one dequantized row */
static size_t g_row_bytes;

static void cuda_row_to_f32(si_backend *be, const si_tensor *w, uint64_t row, float *out) {
    (void)be;
    void *dw = device_copy(w);
    if (!dw) return;
    const size_t need = (size_t)w->ne[0] * sizeof(float);
    char msg[256];
    if (g_row_bytes < need) {
        if (g_row) sicu_free(g_row);
        g_row = NULL;
        g_row_bytes = 0;
        if (sicu_malloc((void **)&g_row, need) != SICU_OK) goto fail;
        g_row_bytes = need;
    }
    const int64_t r = (int64_t)row;
    if (sicu_row_to_f32(w->type, dw, (int64_t)w->ne[0], &r, 1, g_row, NULL) != SICU_OK ||
        sicu_memcpy_d2h(out, g_row, need, NULL) != SICU_OK || sicu_stream_sync(NULL) != SICU_OK)
        goto fail;
    return;
fail:
    sicu_last_error(msg, sizeof msg);
    si_set_err("cuda row_to_f32: %s", msg);
}

static si_backend g_cuda_backend = {
    .name = "cuda",
    .loc = SI_LOC_HOST,
    .gemv = cuda_gemv,
    .row_to_f32 = cuda_row_to_f32,
};

/* The backend for device `device`, or NULL (message in si_errstr()). */
__attribute__((visibility("default"))) si_backend *si_backend_cuda(int device) {
    if (sicu_init(device) != SICU_OK) {
        char msg[256];
        sicu_last_error(msg, sizeof msg);
        si_set_err("cuda backend: %s", msg);
        return NULL;
    }
    return &g_cuda_backend;
}

/* Free every uploaded weight copy. */
__attribute__((visibility("default"))) void si_backend_cuda_release(void) {
    for (int i = 0; i < g_ntab; i++) sicu_free(g_tab[i].dev);
    g_ntab = 0;
    g_last = 0;
    if (g_row) sicu_free(g_row);
    g_row = NULL;
    g_row_bytes = 0;
}
