/* Test infrastructure only (the CPU checker for the CUDA path).
   C restatement of the reference engine's float tier (--fixed off,
   --fastfp off) for the MTP speculative-decoding step of KunMoe.
   Every function cites the reference file:line it follows; the pins are
   the golden vectors produced by the reference itself (tests/golden). */
#ifndef LZ98_ORACLE_H
#define LZ98_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct LzoModel LzoModel;
typedef struct LzoState LzoState;

LzoModel *lzo_open(const char *dir, char *err, int errlen);
void lzo_free(LzoModel *m);
/* vocab, hidden, n_layers, kda heads, key dim, latent, experts, top_k,
   shared width, head_dim, n_heads, n_kv_heads, rotary_dim, seq_len. */
void lzo_info(const LzoModel *m, int *o);

LzoState *lzo_state_new(const LzoModel *m, int seq_len, int spec_k_max);
void lzo_state_free(LzoState *s);
void lzo_state_reset(LzoState *s);
void lzo_get_positions(const LzoState *s, int *mtp_pos, int *ssm_slot, int *ring_depth);
void lzo_set_positions(LzoState *s, int mtp_pos, int ssm_slot);
void lzo_set_chain(LzoState *s, const float *chain);
void lzo_get_chain(const LzoState *s, float *chain);

/* Body forwards (src/forward.c:1619-1837). */
int lzo_forward(const LzoModel *m, LzoState *s, const int *tok, int n, int pos0,
                int advance_ring, float *hidden_out, float *logits_out);
int lzo_mtp_draft(const LzoModel *m, LzoState *s, int tok, int pos, float *logits);
int lzo_mtp_prefill(const LzoModel *m, LzoState *s, const float *hidden,
                    const int *next, int n, int pos0);

int lzo_generate(const LzoModel *m, LzoState *s, const int *prompt, int n_prompt,
                 int max_new, int spec_k, float temp, float topp,
                 unsigned long long seed, int *out_tok, int out_cap, int *out_n,
                 int *rounds, int round_cap, int *n_rounds);
int lzo_generate_pm(const LzoModel *m, LzoState *s, const int *prompt, int n_prompt,
                    int max_new, int spec_k, float temp, float topp,
                    unsigned long long seed, float p_min, int n_min,
                    int *out_tok, int out_cap, int *out_n,
                    int *rounds, int round_cap, int *n_rounds);

/* Op-level restatements. */
float lzo_exp(float x);
float lzo_rsqrt(float x);
float lzo_sigmoid(float x);
void lzo_quantize_q8(const float *x, int n, int gs, signed char *q, float *s);
void lzo_matmul_q8(float *o, const signed char *xq, const float *xqs,
                   const signed char *wq, const float *ws, int gs,
                   int in_dim, int out_dim, int nt);
void lzo_rmsnorm(float *o, const float *x, const float *w, int n, float eps);
void lzo_recur_step(float *out, const signed char *sq_in, signed char *sq_out,
                    const signed char *sl_in, signed char *sl_out,
                    const float *ss_in, float *ss_out,
                    const float *q, const float *k, const float *v,
                    const float *g, float beta, int kd, int vd);
void lzo_moe_route(const float *logits, const float *bias, int n_experts,
                   int top_k, int sigmoid, int renorm, int *idx, float *w);
int lzo_argmax(const float *x, int n);
int lzo_argmax_p1(const float *logits, int n, float *p1);
void lzo_target_dist(float temp, float topp, float *logits, int n, float *out_p);
int lzo_spec_accept(const int *draft, const int *targ, int n, int bonus, int *out);
int lzo_spec_accept_temp(const float *p, const float *q, int x, int vocab,
                         float u, unsigned long long *rng, int *acc);
float lzo_random_f32(unsigned long long *state);

#ifdef __cplusplus
}
#endif
/* Logits of n final-normed hidden rows over vocabulary rows
   [v0, v0 + nv) of the tied lm_head. */
int lzo_lm_head_cols(const LzoModel *m, const float *hidden, int n, int v0, int nv, float *out);

/* The RoPE table [seq_len][rot/2][cos, sin] of the MTP attention. */
void lzo_rope_table(float theta, int rot, int seq_len, float *out);

#endif
