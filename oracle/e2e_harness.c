/* TEST INFRASTRUCTURE ONLY: drives the reference's own engine
 * (si_model_load / si_engine_forward, src/model.c, src/engine.c) with every
 * layer on either the reference CPU backend or the CUDA backend adapter
 * (siphon_b200/csrc/backend_cuda.c), for end-to-end parity tests. Built with
 * the reference sources into _ref/libsiphon_e2e.so (oracle/Makefile). */
#include "siphon/engine.h"
#include "siphon/kernels.h"
#include "siphon/model.h"

si_backend *si_backend_cuda(int device);
void si_backend_cuda_release(void);

typedef struct {
    si_model *m;
    si_engine *e;
    int cuda;
} e2e;

#define E2E_API __attribute__((visibility("default")))

E2E_API const char *e2e_error(void) { return si_errstr(); }

static int g_mode = -1;   /* host kernel mode fixed by the first open */

E2E_API const char *e2e_kern_impl(void) { return si_kern_impl_name(); }

/* use_cuda: 0 = reference CPU backend for every layer, 1 = CUDA backend.
 * The output head stays on the CPU backend in both (src/engine.c:393).
 * scalar: 1 = the reference's portable scalar kernels for all host work
 * (its SI_SCALAR switch, src/kernels.c:80-83), 0 = its default dispatch
 * (AVX2 on x86). The reference reads the switch once, so the first open of
 * the process fixes it. */
E2E_API int e2e_open(const char *path, int use_cuda, int device, int n_ctx, int threads, int scalar,
                     void **out) {
    if (g_mode < 0) {
        if (scalar) setenv("SI_SCALAR", "1", 1);
        else unsetenv("SI_SCALAR");
        si_kern_init();
        g_mode = scalar ? 1 : 0;
    } else if (g_mode != (scalar ? 1 : 0)) {
        si_set_err("e2e: host kernel mode was fixed to %s by the first open", g_mode ? "scalar" : "dispatch");
        return SI_EINVAL;
    }
    e2e *h = calloc(1, sizeof *h);
    int rc = si_model_load(path, &h->m);
    if (rc != SI_OK) { free(h); return rc; }
    if (use_cuda) {
        si_backend *be = si_backend_cuda(device);
        if (!be) { si_model_free(h->m); free(h); return SI_EIO; }
        for (uint32_t il = 0; il < h->m->h.n_layer; il++) h->m->layer_be[il] = be;
        h->cuda = 1;
    }
    rc = si_engine_create(h->m, n_ctx, threads, &h->e);
    if (rc != SI_OK) { si_model_free(h->m); free(h); return rc; }
    *out = h;
    return SI_OK;
}

E2E_API const float *e2e_forward(void *hp, uint32_t token) {
    e2e *h = hp;
    return si_engine_forward(h->e, token);
}

E2E_API uint32_t e2e_n_vocab(void *hp) { return ((e2e *)hp)->m->h.n_vocab; }

E2E_API void e2e_close(void *hp) {
    e2e *h = hp;
    if (!h) return;
    si_engine_free(h->e);
    si_model_free(h->m);
    if (h->cuda) si_backend_cuda_release();
    free(h);
}
