/* Reference-side binding of the GPU library: the file a maintainer of the
   reference adds next to src/generate.c to send the speculative round of
   its generation loop (src/generate.c:1953-1966) to a B200.
 
   The reference keeps its own symbols: liblz98gpu.so is opened at run time
   (dlopen, RTLD_LOCAL) and its entry points are taken by dlsym, so the
   reference's CPU lz_spec_round stays what its own objects call and the
   gpu_* functions below reach the GPU.  The caller's LZSampler
   (src/sampler.h:176-186) passes through unchanged: lz98_gpu.h declares
   the same layout and defers to the reference's definition when sampler.h
   was included first.

   Build inside the reference tree:
       cc -std=c99 -I<repo>/include -I<reference>/src -c lz98_gpu_shim.c
   and link the reference with -ldl.  Without the reference's sampler.h on
   the include path the shim builds against lz98_gpu.h alone. */
#define _POSIX_C_SOURCE 200809L
#include <dlfcn.h>
#include <stdio.h>
#include <string.h>

#if defined(__has_include)
#if __has_include("sampler.h")
#include "sampler.h"           /* the reference's LZSampler, when built in its tree */
#endif
#endif
#include "lz98_gpu.h"
#include "lz98_gpu_shim.h"

#define SHIM_TEMP_FLOOR 1e-3f  /* LZ_TEMP_FLOOR, src/sampler.h:130 */

static struct {
    void *so;
    LZModel *model;
    LZRunState *state;
    int (*open)(LZModel **, const char *, char *, int);
    void (*free_model)(LZModel *);
    int (*state_alloc)(LZRunState **, const LZModel *, int, int, char *, int);
    void (*state_free)(LZRunState *);
    int (*set_sampler)(LZRunState *, int, float, float, uint64_t);
    int (*get_sampler)(const LZRunState *, int, float *, float *, uint64_t *);
    int (*prefill)(const LZModel *, LZRunState *, int, const int *, int, int *, char *, int);
    int (*round)(const LZModel *, LZRunState *, int, int, int, float, int, const LZSampler *, int, int,
                 int *, int *, int *, int *, char *, int);
    int (*round_temp)(const LZModel *, LZRunState *, int, int, int, float, int, LZSampler *, int, int,
                      int *, int *, int *, int *, char *, int);
    int (*accept)(const int *, const int *, int, int, int *);
    int (*accept_temp)(const float *, const float *, int, int, float, uint64_t *, int *);
} G;

static void shim_err(char *err, int errlen, const char *what, const char *detail) {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s%s%s", what, detail ? ": " : "", detail ? detail : "");
}

/* dlsym into a function pointer without a data-to-function cast warning */
static int take(void *dst, const char *name, char *err, int errlen) {
    void *p = dlsym(G.so, name);
    if (!p) {
        shim_err(err, errlen, "symbol missing in the GPU library", name);
        return LZ98_ERR_NULL_ARG;
    }
    memcpy(dst, &p, sizeof p);
    return 0;
}

int gpu_load(const char *so_path, char *err, int errlen) {
    if (G.so) return 0;
    G.so = dlopen(so_path, RTLD_NOW | RTLD_LOCAL);
    if (!G.so) {
        shim_err(err, errlen, "cannot open the GPU library", dlerror());
        return LZ98_ERR_NULL_ARG;
    }
    if (take(&G.open, "lz_open", err, errlen) || take(&G.free_model, "lz_free", err, errlen) ||
        take(&G.state_alloc, "lz_state_alloc", err, errlen) ||
        take(&G.state_free, "lz_state_free", err, errlen) ||
        take(&G.set_sampler, "lz_seq_set_sampler", err, errlen) ||
        take(&G.get_sampler, "lz_seq_get_sampler", err, errlen) ||
        take(&G.prefill, "lz_seq_prefill", err, errlen) || take(&G.round, "lz_spec_round", err, errlen) ||
        take(&G.round_temp, "lz_spec_round_temp", err, errlen) ||
        take(&G.accept, "lz_spec_accept", err, errlen) ||
        take(&G.accept_temp, "lz_spec_accept_temp", err, errlen)) {
        dlclose(G.so);
        memset(&G, 0, sizeof G);
        return LZ98_ERR_NULL_ARG;
    }
    return 0;
}

int gpu_open(const char *model_dir, int seq_len, int spec_k_max, char *err, int errlen) {
    int rc;
    if (!G.so) {
        shim_err(err, errlen, "gpu_load first", NULL);
        return LZ98_ERR_NULL_ARG;
    }
    rc = G.open(&G.model, model_dir, err, errlen);
    if (rc) return rc;
    return G.state_alloc(&G.state, G.model, seq_len, spec_k_max, err, errlen);
}

void gpu_close(void) {
    if (G.state) G.state_free(G.state);
    if (G.model) G.free_model(G.model);
    G.state = NULL;
    G.model = NULL;
}

/* The prompt side of the reference loop (capture prefill of the prompt,
   MTP prompt prefill, capture forward of the last token and the first
   anchor sampled with the caller's sampler, src/generate.c:2841-2900) in
   one call; the caller's generator advances as the reference's would. */
int gpu_prefill(const int *prompt, int n_prompt, LZSampler *samp, int *anchor, char *err, int errlen) {
    int rc;
    float t = 0.0f, p = 0.0f;
    uint64_t rng = 0;
    if (samp) {
        rc = G.set_sampler(G.state, 0, samp->p.temperature, samp->p.topp, samp->rng_state);
        if (rc) return rc;
    }
    rc = G.prefill(G.model, G.state, 0, prompt, n_prompt, anchor, err, errlen);
    if (rc || !samp) return rc;
    rc = G.get_sampler(G.state, 0, &t, &p, &rng);
    if (!rc) samp->rng_state = rng;
    return rc;
}

/* Drop-in for the lz_spec_round / lz_spec_round_temp calls of the
   reference loop (src/generate.c:1953-1966): greedy at the temperature
   floor, else the coupled temperature round, which advances
   samp->rng_state. */
int gpu_spec_round(int anchor, int anchor_pos, int k, float p_min, int n_min, LZSampler *samp, int *out,
                   int *n_accept, int *new_pos, int *k_eff, char *err, int errlen) {
    if (samp && samp->p.temperature > SHIM_TEMP_FLOOR)
        return G.round_temp(G.model, G.state, anchor, anchor_pos, k, p_min, n_min, samp, 0, 0, out, n_accept,
                            new_pos, k_eff, err, errlen);
    return G.round(G.model, G.state, anchor, anchor_pos, k, p_min, n_min, samp, 0, 0, out, n_accept, new_pos,
                   k_eff, err, errlen);
}

int gpu_spec_accept(const int *draft, const int *targ, int n_draft, int bonus, int *out) {
    return G.accept(draft, targ, n_draft, bonus, out);
}

int gpu_spec_accept_temp(const float *p, const float *q, int x, int vocab, float u, uint64_t *rng,
                         int *out_accepted) {
    return G.accept_temp(p, q, x, vocab, u, rng, out_accepted);
}
