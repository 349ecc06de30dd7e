/* The reference-side shim's functions (lz98_gpu_shim.c).  Include after
   the reference's sampler.h or after lz98_gpu.h (for LZSampler). */
#ifndef LZ98_GPU_SHIM_H
#define LZ98_GPU_SHIM_H
#include <stdint.h>

int  gpu_load(const char *so_path, char *err, int errlen);
int  gpu_open(const char *model_dir, int seq_len, int spec_k_max, char *err, int errlen);
void gpu_close(void);
int  gpu_prefill(const int *prompt, int n_prompt, LZSampler *samp, int *anchor, char *err, int errlen);
int  gpu_spec_round(int anchor, int anchor_pos, int k, float p_min, int n_min, LZSampler *samp, int *out,
                    int *n_accept, int *new_pos, int *k_eff, char *err, int errlen);
int  gpu_spec_accept(const int *draft, const int *targ, int n_draft, int bonus, int *out);
int  gpu_spec_accept_temp(const float *p, const float *q, int x, int vocab, float u, uint64_t *rng,
                          int *out_accepted);
#endif
