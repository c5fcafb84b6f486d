/* TEST INFRASTRUCTURE ONLY: drives the reference's own engine
 * (si_model_load / si_engine_forward, src/model.c, src/engine.c) with every
 * matrix product on either the reference CPU backend or the CUDA backend
 * adapter (siphon_b200/csrc/backend_cuda.c), for end-to-end parity tests.
 * Built with the reference sources into _ref/libsiphon_e2e.so
 * (oracle/Makefile).
 *
 * The reference's forward pass takes the embedding lookup and the output
 * head from si_backend_cpu() directly (src/engine.c:302, 393) instead of
 * from a per-model backend. The Makefile compiles src/engine.c (and only that
 * file) with si_backend_cpu renamed to e2e_engine_backend, so those two call
 * sites land here: they get the CUDA backend in a CUDA run and the CPU backend
 * otherwise. This stands in for the two-line source change a maintainer makes
 * (INTEGRATION.md); the reference's sources are compiled unmodified. */
#include "siphon/engine.h"
#include "siphon/kernels.h"
#include "siphon/model.h"

#include <stdlib.h>
#include <string.h>

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
static si_backend *g_engine_be;   /* backend of engine.c's embedding and head sites */

/* engine.c's si_backend_cpu() at src/engine.c:302 (embedding row) and :393
 * (output head) */
si_backend *e2e_engine_backend(void) { return g_engine_be ? g_engine_be : si_backend_cpu(); }

E2E_API const char *e2e_kern_impl(void) { return si_kern_impl_name(); }

/* use_cuda: 0 = reference CPU backend for every product, 1 = CUDA backend for
 * every layer's products, the embedding lookup and the output head.
 * scalar: 1 = the reference's portable scalar kernels for all host work
 * (its SI_SCALAR switch, src/kernels.c:80-83), 0 = its default dispatch
 * (AVX2 on x86). The reference reads the switch once, so the first open of
 * the process fixes it. One engine at a time may be open with use_cuda. */
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
    g_engine_be = h->cuda ? h->m->layer_be[0] : NULL;
    si_set_err("%s", "");
    const float *y = si_engine_forward(h->e, token);
    g_engine_be = NULL;
    /* the backend slots return void and report through si_set_err; a failed
     * product leaves stale outputs, so check the message like a careful
     * caller of the reference would */
    if (y && h->cuda && strncmp(si_errstr(), "cuda", 4) == 0) return NULL;
    return y;
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
