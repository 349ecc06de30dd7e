#define _POSIX_C_SOURCE 199309L
/* Test infrastructure: a small driver over the UNMODIFIED reference engine,
   compiled into oracle/_ref/liblz98ref.so together with the reference
   sources.  It exists because the reference's own speculative path is only
   reachable through lz_generate_call, which needs a tokenizer; this file
   replays that loop on token ids with the reference's public calls.

   The loop follows lz_generate_call (src/generate.c:2781-3091) and
   lz_generate_spec_round (src/generate.c:1822-2100) with no EOS, no stop
   strings and no cancellation: prompt capture-prefill
   (lz_forward_batch_capture), MTP prompt prefill (lz_mtp_prefill), then
   speculative rounds while the budget allows one (round_k clamp of
   src/generate.c:3013-3024), then plain per-token steps.

   The arithmetic tier is pinned as the parity tier: --fixed off
   (lz_float_ref_select("off")), --fastfp off (RN, no FTZ) and the kernel
   tier passed by the caller (LZ_KERNEL_AVX2 = 7 or LZ_KERNEL_REF = 1).
   The tier is process-global in the reference; the last rd_open wins. */
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "forward.h"
#include "llama_zh.h"
#include "model.h"
#include "ops.h"
#include "sampler.h"

typedef struct {
    LZModel m;
    LZRunState s;
    int have_m, have_s;
} RdHandle;

/* The rounds' two test-only switches, passed unchanged to lz_spec_round /
   lz_spec_round_temp by the generation loop below: debug_break_rollback
   (the reference's known-bad control, src/generate.c:827-844: a rejected
   round leaves the state ring where the full verify left it) and
   debug_skip_catchup (src/generate.c:976-982).  Process-global; 0 by
   default. */
static int rd_dbg_break_rollback = 0, rd_dbg_skip_catchup = 0;

/* The state's RoPE table (s->rope_cs, [seq_len][rot/2][cos, sin], built by
   lz_rope_build_table, src/forward_rope.c:178-187) into out. */
int rd_rope_table(void *vh, float *out, int n) {
    RdHandle *h = (RdHandle *)vh;
    int need = h->s.seq_len * h->m.config.rotary_dim;
    if (!h->s.rope_cs || n < need) return -1;
    memcpy(out, h->s.rope_cs, sizeof(float) * (size_t)need);
    return need;
}

void rd_set_round_debug(int break_rollback, int skip_catchup) {
    rd_dbg_break_rollback = break_rollback;
    rd_dbg_skip_catchup = skip_catchup;
}

static double rd_now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

void rd_set_tier(int kernel) {
    lz_float_ref_select("off");
    lz_fastfp_select("off");
    lz_kernel_select(kernel);
}

/* The reference's stock arithmetic, its CLI defaults (cli_main.c:483,
   cli_main.c:531): --fixed all (the shipping fixed-point tier) and --fastfp
   on (round toward zero, flush to zero inside the engine's float regions,
   which restore the caller's MXCSR on exit, ops_quant.c:2015-2050), with
   the given kernel tier.  Used only to time the reference as shipped; its
   tokens differ from the parity tier's by design.  Process-global like
   rd_set_tier: it holds for every handle until the next call of either. */
void rd_set_stock_tier(int kernel) {
    lz_float_ref_select("all");
    lz_fastfp_select("on");
    lz_kernel_select(kernel);
}

void *rd_open(const char *dir, int seq_len, int spec_k_max, int nt_cap,
              int kernel, char *err, int errlen) {
    RdHandle *h = (RdHandle *)calloc(1, sizeof(RdHandle));
    if (!h) return NULL;
    rd_set_tier(kernel);
    if (lz_open(&h->m, dir, err, errlen) != 0) { free(h); return NULL; }
    h->have_m = 1;
    if (lz_read_weights(&h->m, err, errlen) != 0) {
        lz_free(&h->m); free(h); return NULL;
    }
    if (lz_state_alloc(&h->s, &h->m, seq_len, spec_k_max, err, errlen) != 0) {
        lz_free(&h->m); free(h); return NULL;
    }
    h->have_s = 1;
    if (nt_cap > 0) h->s.nt_cap = nt_cap;
    return h;
}

void rd_session_end_owned(void *vh);

void rd_close(void *vh) {
    RdHandle *h = (RdHandle *)vh;
    if (!h) return;
    rd_session_end_owned(vh);
    if (h->have_s) lz_state_free(&h->s);
    if (h->have_m) lz_free(&h->m);
    free(h);
}

void rd_reset(void *vh) {
    RdHandle *h = (RdHandle *)vh;
    lz_state_reset(&h->s, &h->m);
}

/* Selected config words: vocab, hidden, n_layers, ring depth, mtp_pos,
   ssm_slot, kda heads, key dim, latent, experts, top_k, shared width,
   head_dim, n_heads, n_kv_heads, rotary_dim. */
void rd_info(void *vh, int *o) {
    RdHandle *h = (RdHandle *)vh;
    const LZModelConfig *c = &h->m.config;
    o[0] = c->vocab_size; o[1] = c->hidden_size; o[2] = c->n_layers;
    o[3] = h->s.ssm_ring_depth; o[4] = h->s.mtp_pos; o[5] = h->s.ssm_slot;
    o[6] = c->lin_n_v_heads; o[7] = c->lin_key_dim; o[8] = c->moe_latent_dim;
    o[9] = c->num_experts; o[10] = c->num_experts_per_token;
    o[11] = c->moe_shared_width; o[12] = c->head_dim; o[13] = c->n_heads;
    o[14] = c->n_kv_heads; o[15] = c->rotary_dim;
}

void rd_set_positions(void *vh, int mtp_pos, int ssm_slot) {
    RdHandle *h = (RdHandle *)vh;
    if (mtp_pos >= 0) h->s.mtp_pos = mtp_pos;
    if (ssm_slot >= 0) h->s.ssm_slot = ssm_slot;
}

/* Body forward of n tokens with capture of the final-normed hidden rows.
   Returns 0 on success. */
int rd_batch_capture(void *vh, const int *tok, int n, int pos0, float *hidden) {
    RdHandle *h = (RdHandle *)vh;
    return lz_forward_batch_capture(&h->m, &h->s, tok, n, pos0, hidden) ? 0 : 1;
}

/* Single-token forward with mtp_chain capture; copies logits and chain. */
int rd_forward_capture(void *vh, int tok, int pos, float *logits, float *chain) {
    RdHandle *h = (RdHandle *)vh;
    float *lg = lz_forward_capture(&h->m, &h->s, tok, pos);
    if (!lg) return 1;
    if (logits) memcpy(logits, lg, sizeof(float) * (size_t)h->m.config.vocab_size);
    if (chain && h->s.mtp_chain)
        memcpy(chain, h->s.mtp_chain, sizeof(float) * (size_t)h->m.config.hidden_size);
    return 0;
}

/* Verify forward of n tokens: every row's logits and captured hidden. */
int rd_forward_verify(void *vh, const int *tok, int n, int pos0,
                      float *logits, float *hidden) {
    RdHandle *h = (RdHandle *)vh;
    const LZModelConfig *c = &h->m.config;
    if (lz_forward_verify(&h->m, &h->s, tok, n, pos0) != 0) return 1;
    if (logits) memcpy(logits, h->s.mtp_logits, sizeof(float) * (size_t)n * c->vocab_size);
    if (hidden) memcpy(hidden, h->s.mtp_verify_hidden, sizeof(float) * (size_t)n * c->hidden_size);
    return 0;
}

int rd_mtp_draft(void *vh, int tok, int pos, float *logits, float *chain) {
    RdHandle *h = (RdHandle *)vh;
    float *lg = lz_mtp_draft_step(&h->m, &h->s, tok, pos);
    if (!lg) return 1;
    if (logits) memcpy(logits, lg, sizeof(float) * (size_t)h->m.config.vocab_size);
    if (chain) memcpy(chain, h->s.mtp_chain, sizeof(float) * (size_t)h->m.config.hidden_size);
    return 0;
}

int rd_mtp_prefill(void *vh, const float *hidden, const int *next, int n, int pos0) {
    RdHandle *h = (RdHandle *)vh;
    return lz_mtp_prefill(&h->m, &h->s, hidden, next, n, pos0);
}

void rd_set_chain(void *vh, const float *chain) {
    RdHandle *h = (RdHandle *)vh;
    memcpy(h->s.mtp_chain, chain, sizeof(float) * (size_t)h->m.config.hidden_size);
}

/* A generation on token ids, split so that the decode can run in bounded
   slices: rd_session_begin resets the state and prefills the prompt,
   rd_session_decode runs the decode loop until max_tokens more tokens have
   been emitted, the budget (n_prompt + max_new positions) is used up, or
   budget_ms of wall time has passed (checked between rounds, 0 = no
   limit), and can be called again to go on where it stopped;
   rd_session_end frees the sampler.  rd_generate_pm is begin + one
   unlimited decode + end.

   temp <= 0 runs the greedy rounds (lz_spec_round), temp > 0 the coupled
   rounds (lz_spec_round_temp) with top-p `topp` and the sampler seeded
   with `seed`.  spec_k = 0 disables speculation (plain per-token decode).
   A discarded draft (n_emit == 0, p_min / n_min) emits nothing and forces
   a fresh capture next round (src/generate.c:1972-2080).
   out_tok receives every emitted token of the call in order (cap
   out_cap); rounds receives (k_eff, n_accept) per speculative round (cap
   round_cap).  Return 0 on success, else a positive code. */
typedef struct {
    LZSampler samp;
    void *owner;
    int active, pos, token, max_pos, have_seed, spec_k, n_min;
    float temp, p_min;
} RdSession;

static RdSession rd_sess;   /* one session per process (the tier is process-global too) */

void rd_session_end(void *vh) {
    (void)vh;
    if (rd_sess.active) lz_sampler_free(&rd_sess.samp);
    rd_sess.active = 0;
}

/* rd_close's part: the session of this handle, if any, ends with it */
void rd_session_end_owned(void *vh) {
    if (rd_sess.active && rd_sess.owner == vh) rd_session_end(vh);
}

int rd_session_begin(void *vh, const int *prompt, int n_prompt, int max_new,
                     int spec_k, float temp, float topp, unsigned long long seed,
                     float p_min, int n_min, double *prefill_ms) {
    RdHandle *h = (RdHandle *)vh;
    const LZModel *m = &h->m;
    LZRunState *s = &h->s;
    const LZModelConfig *c = &m->config;
    LZSampleParams sp;
    RdSession *q = &rd_sess;
    double t0 = rd_now_ms();

    rd_session_end(vh);
    lz_sample_defaults(&sp);
    sp.temperature = temp > 0.0f ? temp : 0.0f;
    sp.topp = topp;
    sp.topk = 0;
    sp.minp = 0.0f;
    sp.presence_penalty = 0.0f;
    sp.frequency_penalty = 0.0f;
    sp.repetition_penalty = 1.0f;
    sp.repeat_last_n = 0;
    sp.think_temp_enabled = 0;
    if (lz_sampler_init(&q->samp, c->vocab_size, &sp, (lz_u64)seed) != 0) return 1;
    q->active = 1;
    q->owner = vh;
    q->spec_k = spec_k;
    q->temp = temp;
    q->p_min = p_min;
    q->n_min = n_min;
    q->have_seed = 0;

    lz_state_reset(s, m);
    q->max_pos = n_prompt + max_new;
    if (q->max_pos > s->seq_len) q->max_pos = s->seq_len;
    if (q->max_pos < n_prompt + 1) q->max_pos = n_prompt + 1;

    if (n_prompt > 1) {
        if (spec_k > 0) {
            float *hb = (float *)malloc(sizeof(float) * (size_t)(n_prompt - 1) *
                                        (size_t)c->hidden_size);
            if (!hb) return 1;
            if (!lz_forward_batch_capture(m, s, prompt, n_prompt - 1, 0, hb)) {
                free(hb); return 2;
            }
            if (lz_mtp_prefill(m, s, hb, prompt + 1, n_prompt - 1, s->mtp_pos) != 0) {
                free(hb); return 3;
            }
            s->mtp_pos = s->mtp_pos + (n_prompt - 1);
            free(hb);
        } else {
            if (!lz_forward_batch(m, s, prompt, n_prompt - 1, 0)) return 2;
        }
    }
    if (prefill_ms) *prefill_ms = rd_now_ms() - t0;
    q->pos = n_prompt - 1;
    q->token = prompt[n_prompt - 1];
    return 0;
}

int rd_session_decode(void *vh, int max_tokens, double budget_ms,
                      int *out_tok, int out_cap, int *out_n,
                      int *rounds, int round_cap, int *n_rounds, double *elapsed_ms) {
    RdHandle *h = (RdHandle *)vh;
    const LZModel *m = &h->m;
    LZRunState *s = &h->s;
    RdSession *q = &rd_sess;
    int rc = 0, n_out = 0, nr = 0;
    double t0 = rd_now_ms();
    char err[256];

    if (!q->active || q->owner != vh) return 1;
    while (q->pos < q->max_pos - 1 && n_out < max_tokens &&
           (budget_ms <= 0.0 || rd_now_ms() - t0 < budget_ms)) {
        int round_k = 0;
        if (q->spec_k > 0) {
            round_k = q->spec_k;
            if (round_k > q->max_pos - 3 - q->pos) round_k = q->max_pos - 3 - q->pos;
        }
        if (round_k > 0) {
            int anchor, anchor_pos, n_accept = 0, new_pos = 0, k_eff = 0, n_emit, ei;
            int out[LZ_SPEC_K_MAX + 1];
            if (q->have_seed) {
                anchor = q->token;
                anchor_pos = q->pos - 1;
            } else {
                float *lg = lz_forward_capture(m, s, q->token, q->pos);
                if (!lg) { rc = 4; goto out; }
                anchor_pos = q->pos;
                anchor = lz_sample_ex(&q->samp, lg, NULL, 0);
                lz_sampler_observe(&q->samp, anchor);
                if (n_out < out_cap) out_tok[n_out] = anchor;
                n_out++;
            }
            if (q->temp > 0.0f)
                n_emit = lz_spec_round_temp(m, s, anchor, anchor_pos, round_k,
                                            q->p_min, q->n_min, &q->samp, rd_dbg_break_rollback,
                                            rd_dbg_skip_catchup, out, &n_accept,
                                            &new_pos, &k_eff, err, (int)sizeof err);
            else
                n_emit = lz_spec_round(m, s, anchor, anchor_pos, round_k,
                                       q->p_min, q->n_min, &q->samp, rd_dbg_break_rollback,
                                       rd_dbg_skip_catchup, out, &n_accept,
                                       &new_pos, &k_eff, err, (int)sizeof err);
            if (n_emit < 0) { rc = -n_emit; goto out; }
            if (nr < round_cap) { rounds[2 * nr] = k_eff; rounds[2 * nr + 1] = n_accept; }
            nr++;
            q->have_seed = (n_emit > 0);
            if (n_emit > 0) {
                for (ei = 0; ei <= n_accept; ei++) {
                    lz_sampler_observe(&q->samp, out[ei]);
                    if (n_out < out_cap) out_tok[n_out] = out[ei];
                    n_out++;
                }
            }
            q->pos = new_pos + 1;
            q->token = out[n_accept];
            continue;
        }
        {
            float *lg = lz_forward(m, s, q->token, q->pos);
            int next;
            if (!lg) { rc = 5; goto out; }
            next = lz_sample_ex(&q->samp, lg, NULL, 0);
            lz_sampler_observe(&q->samp, next);
            if (n_out < out_cap) out_tok[n_out] = next;
            n_out++;
            q->token = next;
            q->pos++;
        }
    }
out:
    if (elapsed_ms) *elapsed_ms = rd_now_ms() - t0;
    *out_n = n_out;
    *n_rounds = nr;
    return rc;
}

int rd_generate_pm(void *vh, const int *prompt, int n_prompt, int max_new,
                   int spec_k, float temp, float topp, unsigned long long seed,
                   float p_min, int n_min,
                   int *out_tok, int out_cap, int *out_n,
                   int *rounds, int round_cap, int *n_rounds,
                   double *elapsed_ms, double *prefill_ms) {
    double pf = 0.0, dec = 0.0;
    int rc = rd_session_begin(vh, prompt, n_prompt, max_new, spec_k, temp, topp, seed,
                              p_min, n_min, &pf);
    *out_n = 0;
    *n_rounds = 0;
    if (rc == 0)
        rc = rd_session_decode(vh, 1 << 30, 0.0, out_tok, out_cap, out_n,
                               rounds, round_cap, n_rounds, &dec);
    rd_session_end(vh);
    if (prefill_ms) *prefill_ms = pf;
    if (elapsed_ms) *elapsed_ms = pf + dec;
    return rc;
}

int rd_generate(void *vh, const int *prompt, int n_prompt, int max_new,
                int spec_k, float temp, float topp, unsigned long long seed,
                int *out_tok, int out_cap, int *out_n,
                int *rounds, int round_cap, int *n_rounds,
                double *elapsed_ms, double *prefill_ms) {
    return rd_generate_pm(vh, prompt, n_prompt, max_new, spec_k, temp, topp, seed, 0.0f, 0,
                          out_tok, out_cap, out_n, rounds, round_cap, n_rounds,
                          elapsed_ms, prefill_ms);
}

/* ---- op-level entry points (plain pointers; the tensor is built here) -- */

void rd_matmul_q8(float *o, const signed char *xq, const float *xqs,
                  const signed char *wq, const float *ws, int gs,
                  int in_dim, int out_dim, int nt) {
    LZTensor w;
    memset(&w, 0, sizeof w);
    w.dtype = LZ_FMT_Q8_0;
    w.n = in_dim * out_dim;
    w.gs = gs;
    w.q = (int8_t *)wq;
    w.scale = (float *)ws;
    lz_matmul_xq_nt(o, NULL, (const int8_t *)xq, xqs, &w, in_dim, out_dim, nt);
}

void rd_quantize_q8(const float *x, int n, int gs, signed char *q, float *s) {
    lz_quantize_q8(x, n, gs, (int8_t *)q, s);
}

float rd_exp(float x) { unsigned f = lz_fpu_float_begin(); float r = lz_exp(x); lz_fpu_float_end(f); return r; }
float rd_rsqrt(float x) { unsigned f = lz_fpu_float_begin(); float r = lz_rsqrt(x); lz_fpu_float_end(f); return r; }
float rd_sigmoid(float x) { unsigned f = lz_fpu_float_begin(); float r = lz_sigmoid(x); lz_fpu_float_end(f); return r; }

void rd_rmsnorm(float *o, const float *x, const float *w, int n, float eps) {
    unsigned f = lz_fpu_float_begin();
    lz_rmsnorm(o, x, w, n, eps);
    lz_fpu_float_end(f);
}

void rd_recur_step(float *out, const signed char *sq_in, signed char *sq_out,
                   const signed char *sl_in, signed char *sl_out,
                   const float *ss_in, float *ss_out,
                   const float *q, const float *k, const float *v,
                   const float *g, float beta, int kd, int vd) {
    unsigned f = lz_fpu_float_begin();
    lz_kda_step(out, (const int8_t *)sq_in, (int8_t *)sq_out,
                (const int8_t *)sl_in, (int8_t *)sl_out, ss_in, ss_out,
                q, k, v, g, beta, kd, vd);
    lz_fpu_float_end(f);
}

void rd_moe_route(const float *logits, const float *bias, int n_experts,
                  int top_k, int sigmoid, int renorm, int *idx, float *w) {
    LZMoeRouteParams rp;
    unsigned f = lz_fpu_float_begin();
    memset(&rp, 0, sizeof rp);
    rp.li_e = 0;
    rp.bias = bias;
    rp.n_experts = n_experts;
    rp.top_k = top_k;
    rp.sigmoid = sigmoid;
    rp.renormalize = renorm;
    rp.tau = 1.0f;
    rp.idx_out = idx;
    rp.w_out = w;
    lz_moe_route(logits, NULL, &rp);
    lz_fpu_float_end(f);
}

int rd_spec_accept(const int *draft, const int *targ, int n, int bonus, int *out) {
    return lz_spec_accept(draft, targ, n, bonus, out);
}

int rd_spec_accept_temp(const float *p, const float *q, int x, int vocab,
                        float u, unsigned long long *rng, int *acc) {
    lz_u64 r = (lz_u64)*rng;
    int t = lz_spec_accept_temp(p, q, x, vocab, u, &r, acc);
    *rng = (unsigned long long)r;
    return t;
}

void rd_target_dist(float temp, float topp, float *logits, int n, float *out_p) {
    LZSampleParams sp;
    LZProbIndex *buf = (LZProbIndex *)malloc(sizeof(LZProbIndex) * (size_t)n);
    unsigned f = lz_fpu_float_begin();
    lz_sample_defaults(&sp);
    sp.temperature = temp; sp.topp = topp; sp.topk = 0; sp.minp = 0.0f;
    lz_target_dist(&sp, logits, n, buf, out_p);
    lz_fpu_float_end(f);
    free(buf);
}

int rd_argmax_p1(const float *logits, int n, float *p1) {
    unsigned f = lz_fpu_float_begin();
    int r = lz_argmax_p1(logits, n, p1);
    lz_fpu_float_end(f);
    return r;
}
