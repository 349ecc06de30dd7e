/* C ABI of the B200-native MTP speculative-decoding step for KunMoe.
 *
 * Drop-in boundary for the reference engine's exports on this path
 * (llama98.def:6-66; prototypes in the reference's src/llama_zh.h and
 * src/forward.h).  Plain pointers and sizes only.  Differences from the
 * reference surface, all forced by the model and the run state living in
 * GPU memory:
 *   - LZModel / LZRunState are opaque handles (the reference's are
 *     by-value structs the caller allocates); lz_open and lz_state_alloc
 *     return them through an out pointer;
 *   - the fields generate.c pokes directly (ssm_slot, mtp_pos, mtp_chain,
 *     mtp_logits, mtp_verify_hidden) are reached through accessors;
 *   - returned float* point into host mirrors owned by the state, valid
 *     until the next call on that state (as in the reference).
 * Error convention as in the reference: round functions return a negative
 * LZErr and fill errbuf; forward functions return NULL or nonzero.
 * One caller per state at a time (src/llama_zh.h:140-143). */
#ifndef LZ98_GPU_H
#define LZ98_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct LZModel LZModel;
typedef struct LZRunState LZRunState;

/* The reference's sampler, field for field (src/sampler.h:140-186), so a
   caller's own LZSampler passes through lz_spec_round / lz_spec_round_temp
   unchanged.  When the reference's sampler.h has been included first
   (its guard LZ_SAMPLER_H), its definitions are used instead.  The rounds
   read p.temperature, p.topp and rng_state (advanced by the temperature
   round), and refuse what the device path does not carry: penalties that
   act (repeat_last_n != 0 with a repetition penalty != 1 or a presence or
   frequency penalty != 0; the reference's assumed-window penalties,
   src/generate.c:517-529), and top-k in (0, vocab) and min-p > 0
   (temperature rounds only; the greedy round reads penalties only, as the
   reference's does).  The think temperature is not read by the rounds. */
#ifndef LZ_SAMPLER_H
typedef struct {
    float prob;
    int   index;
} LZProbIndex;

typedef struct {
    float temperature;
    float temp_think;
    int   think_temp_enabled;
    float topp;
    float minp;
    int   topk;
    float presence_penalty;
    float frequency_penalty;
    float repetition_penalty;
    int   repeat_last_n;
    int   minp_llamacpp;
} LZSampleParams;

typedef struct {
    int            vocab_size;
    LZSampleParams p;
    uint64_t       rng_state;
    LZProbIndex   *probindex;
    unsigned short *counts;
    int           *ring;
    int            cap;
    int            head;
    int            n_win;
} LZSampler;
#endif

/* LZErr codes used on this path, with the values of the reference's
   err.h (src/err.h:19-...), plus four of this library's own from 1000. */
enum {
    LZ98_ERR_OK = 0,
    LZ98_ERR_NULL_ARG = 6,
    LZ98_ERR_ALLOC = 7,          /* LZ_ERR_STATE_ALLOC */
    LZ98_ERR_FORWARD = 20,
    LZ98_ERR_CKPT_EMPTY = 21,
    LZ98_ERR_CKPT_STALE = 22,
    LZ98_ERR_CKPT_SHAPE = 23,
    LZ98_ERR_SPEC_NO_HEAD = 24,
    LZ98_ERR_SPEC_K_RANGE = 25,
    LZ98_ERR_CUDA = 1000,        /* a CUDA call failed, or a device wait gave up */
    LZ98_ERR_MODEL = 1001,       /* model.bin not loadable by this library */
    LZ98_ERR_SIZE = 1002,        /* a request exceeds a fixed limit of this library */
    LZ98_ERR_DEVICE = 1003       /* the current CUDA device is not the model's */
};

/* ---- model: replaces lz_open + lz_read_weights + lz_free
   (src/model.h:1333-1339).  Reads DIR/model.bin ("L98Z" v5-v9 headers,
   scale layouts 0/1/2) and uploads
   every tensor to device memory of the current CUDA device. */
int  lz_open(LZModel **out, const char *dir, char *errbuf, int errlen);
/* The tensors are already resident after lz_open: returns 0 for a valid
   handle (kept so that the reference's open-then-read call order works). */
int  lz_read_weights(LZModel *m, char *errbuf, int errlen);
void lz_free(LZModel *m);
/* (no counterpart in the reference, whose LZModel is a by-value struct the
   caller reads) vocab, hidden, n_layers, kda_heads, key_dim, latent,
   n_experts, top_k, shared_width, head_dim, n_heads, n_kv_heads,
   rotary_dim, seq_len, mtp_ffn, moe_ffn */
void lz_model_info(const LZModel *m, int *out16);
/* Bytes of weights resident in HBM (no counterpart in the reference). */
size_t lz_model_weight_bytes(const LZModel *m);

/* ---- run state: replaces lz_state_alloc / lz_state_reset /
   lz_state_free (src/forward.h:1847-1933).  n_seq independent sequences
   share one allocation (n_seq = 1 is the reference's LZRunState). */
int  lz_state_alloc(LZRunState **out, const LZModel *m, int seq_len,
                    int spec_k_max, char *errbuf, int errlen);
int  lz_state_alloc_batch(LZRunState **out, const LZModel *m, int n_seq,
                          int seq_len, int spec_k_max, char *errbuf, int errlen);
void lz_state_reset(LZRunState *s, const LZModel *m);
void lz_state_free(LZRunState *s);
/* Host mirrors of the LZRunState fields the reference's round loop reads
   and writes directly (mtp_pos, ssm_slot, ssm_ring_depth, mtp_chain;
   src/forward.h:824-1164), for sequence `seq`. */
int  lz_state_get(const LZRunState *s, int seq, int *mtp_pos, int *ssm_slot,
                  int *ring_depth);
int  lz_state_set(LZRunState *s, int seq, int mtp_pos, int ssm_slot);
int  lz_state_get_chain(const LZRunState *s, int seq, float *chain);
int  lz_state_set_chain(LZRunState *s, int seq, const float *chain);

/* ---- forwards of sequence 0 (src/forward.c:1619-1837). */
float *lz_forward(const LZModel *m, LZRunState *s, int token, int pos);
float *lz_forward_capture(const LZModel *m, LZRunState *s, int token, int pos);
float *lz_forward_batch_capture(const LZModel *m, LZRunState *s,
                                const int *tokens, int n, int pos0,
                                float *hidden_out);
/* Verify forward (src/forward.c:1774-1837): logits of every row into the
   state's mtp_logits mirror, captured hidden rows into mtp_verify_hidden
   (the reference's s->mtp_logits and s->mtp_verify_hidden,
   src/forward.h:824-1164, read through the two accessors below). */
int    lz_forward_verify(const LZModel *m, LZRunState *s, const int *tokens,
                         int n, int pos0);
const float *lz_state_mtp_logits(const LZRunState *s);
const float *lz_state_mtp_verify_hidden(const LZRunState *s);

/* ---- MTP draft head of sequence 0 (src/forward_mtp.c:32-144,
   561-642). */
float *lz_mtp_draft_step(const LZModel *m, LZRunState *s, int next_token, int pos);
int    lz_mtp_prefill(const LZModel *m, LZRunState *s, const float *h_body_all,
                      const int *next_tokens, int n, int pos0);
int    lz_mtp_catchup(const LZModel *m, LZRunState *s, const float *h_body_all,
                      const int *next_tokens, int n, int pos0);

/* ---- rounds of sequence 0 (src/llama_zh.h:470-593,
   src/generate.c:694-994 and 1234-1377).  lz_spec_round is the greedy
   round (samp may be NULL; a non-NULL samp with acting penalties is
   refused with -LZ98_ERR_FORWARD, its temperature is not read);
   lz_spec_round_temp the coupled temperature round (temperature above the
   floor, top-p; the refusals listed at LZSampler), which advances
   samp->rng_state as the reference does.  debug_break_rollback is the
   reference's known-bad control (src/generate.c:827-844): a round that
   rejects a draft leaves the state ring where the full verify left it
   instead of rolling it back; debug_skip_catchup skips the MTP catch-up
   (src/generate.c:976-982).  A device wait that gave up during the round
   returns -LZ98_ERR_CUDA; the state is then not usable (free it).
   p_min > 0 stops drafting at the first step whose
   confidence - lz_argmax_p1's probability of the greedy draft, q(x) of a
   sampled one - is below it (that token is not drafted); n_min > 0
   discards a draft of fewer than n_min tokens: the call returns 0 with
   out[0] = anchor, *out_n_accept = 0, *out_new_pos = anchor_pos and
   nothing verified (src/generate.c:421-440, 741-791).  With either set the
   round runs its draft steps one at a time (a host read of each step's
   confidence) instead of as one captured graph. */
int lz_spec_round(const LZModel *m, LZRunState *s, int anchor, int anchor_pos,
                  int k, float p_min, int n_min, const LZSampler *samp,
                  int debug_break_rollback, int debug_skip_catchup,
                  int *out, int *out_n_accept, int *out_new_pos, int *out_k_eff,
                  char *errbuf, int errlen);
int lz_spec_round_temp(const LZModel *m, LZRunState *s, int anchor, int anchor_pos,
                       int k, float p_min, int n_min, LZSampler *samp,
                       int debug_break_rollback, int debug_skip_catchup,
                       int *out, int *out_n_accept, int *out_new_pos, int *out_k_eff,
                       char *errbuf, int errlen);

/* ---- model-free acceptance (src/generate.c:232-349). */
int lz_spec_accept(const int *draft, const int *targ, int n_draft, int bonus, int *out);
int lz_spec_accept_temp(const float *p, const float *q, int x, int vocab, float u,
                        uint64_t *residual_rng, int *out_accepted);

/* ---- batched extension (appended surface, no reference counterpart
   beyond lz_spec_round itself): all n_seq sequences of the state advance
   one greedy round together on the device. */
/* Per-sequence prefill of sequence `seq`: capture-prefill of the prompt,
   MTP prompt prefill, first anchor (greedy) from the forward of the last
   prompt token.  Leaves the sequence ready for rounds; returns the anchor. */
int lz_seq_prefill(const LZModel *m, LZRunState *s, int seq, const int *prompt,
                   int n_prompt, int *out_anchor, char *errbuf, int errlen);
/* Sampler of sequence `seq` (the LZSampler fields the path reads,
   src/sampler.h:145-187): temperature (<= 1e-3 is greedy), top-p, and the
   xorshift64* seed (0 is taken as 1, src/sampler.c:55-60).  Kept across
   lz_state_reset, as the reference keeps its sampler apart from the run
   state.  lz_seq_prefill picks the first anchor with it. */
int lz_seq_set_sampler(LZRunState *s, int seq, float temperature, float topp, uint64_t seed);
/* (no counterpart in the reference, whose caller owns its LZSampler) The
   sampler of sequence `seq` as the device holds it: temperature, top-p and
   the generator state, which lz_seq_prefill's anchor sample and the
   temperature rounds advance.  Any output pointer may be NULL. */
int lz_seq_get_sampler(const LZRunState *s, int seq, float *temperature, float *topp, uint64_t *rng);
/* One round of every sequence with draft depth k (device resident:
   draft k steps, one (k+1)-row verify per sequence, acceptance, ring
   rollback, chain reseed, catch-up): greedy when every sequence's sampler
   is at the temperature floor, temperature rounds when none is (mixed
   batches are refused).  out_tokens (n_seq x (k+1)) and
   out_counts (n_seq) may be NULL, which skips the device-to-host copy. */
int lz_spec_round_batch(const LZModel *m, LZRunState *s, int k,
                        int *out_tokens, int *out_counts, char *errbuf, int errlen);
/* (no counterpart in the reference) Capture the round of depth k into a
   CUDA graph (replayed by later lz_spec_round_batch calls of the same k);
   0 disables graphs. */
int lz_set_graphs(LZRunState *s, int enable);
/* (no counterpart in the reference) Launch every kernel with
   programmatic dependent launch (the default):
   each kernel lets the next one start its prologue - weight prefetch -
   while it finishes; 0 launches them plainly serialised. */
int lz_set_pdl(LZRunState *s, int enable);
/* (no counterpart in the reference) 1: dense int8 GEMMs of more than 8
   token rows on the 5th-generation tensor cores (tcgen05.mma kind::i8 into
   tensor memory); 0 (the default): the warp-level mma.sync kernel.  Both
   give the same bits. */
int lz_set_umma(LZRunState *s, int enable);
/* Whole generation on token ids (the reference's lz_generate_call spec
   loop, src/generate.c:2781-3091, without EOS/stop strings): greedy when
   temp <= 1e-3, else the coupled temperature rounds with top-p `topp`. */
int lz_generate(const LZModel *m, LZRunState *s, const int *prompt, int n_prompt,
                int max_new, int spec_k, float temp, float topp, uint64_t seed,
                int *out_tok, int out_cap, int *out_n, int *rounds, int round_cap,
                int *n_rounds, char *errbuf, int errlen);
/* lz_generate with the rounds' p_min / n_min (a discarded draft emits
   nothing and the next round starts from a fresh capture forward,
   src/generate.c:1972-2080). */
int lz_generate_ex(const LZModel *m, LZRunState *s, const int *prompt, int n_prompt,
                   int max_new, int spec_k, float temp, float topp, uint64_t seed,
                   float p_min, int n_min, int *out_tok, int out_cap, int *out_n,
                   int *rounds, int round_cap, int *n_rounds, char *errbuf, int errlen);

/* The generation loop of sequence 0 continued from body position
   start_pos with the suffix tokens as its prompt, the state NOT reset (the
   reference's lz_generate_resume, src/generate.c:2781-2840, on token ids):
   after lz_prefix_prepare_tokens, start_pos is its *out_start_pos. */
int lz_generate_resume(const LZModel *m, LZRunState *s, int start_pos, const int *suffix, int n_suffix,
                       int max_new, int spec_k, float temp, float topp, uint64_t seed, int *out_tok,
                       int out_cap, int *out_n, int *rounds, int round_cap, int *n_rounds, char *errbuf,
                       int errlen);

/* ---- expert parallelism (no counterpart in the reference, which runs one
   process on one CPU).  The routed experts of every MoE layer are split
   over `world` ranks, one process per GPU: rank r computes experts
   [r E/world, (r+1) E/world) for the pairs of every rank, each rank keeps
   its own sequences.  Per layer the (token, expert) pairs go to their
   expert's owner and the expert outputs come back (NCCL send/recv over
   NVLink, the library bound at run time: the libnccl.so.2 already loaded
   in the process, else the path in LZ98_NCCL, else the system's - a
   process that loads another NCCL itself must do so first); the combine
   keeps the
   reference's selection order, so results are those of one GPU bit for
   bit.  Rank 0 makes the id with lz_ep_unique_id and the caller hands it
   to every rank; every rank then calls lz_ep_init together (collective).
   Every rank must then run the same sequence of forwards (the same
   rounds, prefills of the same lengths): each layer exchanges with every
   peer.  Expert-parallel rounds run eagerly, without graph capture.  A
   stream that does not drain within 60 s aborts the communicator and the
   call returns LZ98_ERR_CUDA.  world <= 8, E divisible by world. */
int lz_ep_unique_id(uint8_t *out128, char *errbuf, int errlen);
int lz_ep_init(LZRunState *s, const uint8_t *id128, int rank, int world, char *errbuf, int errlen);

/* ---- prefix reuse: replaces LZPrefixCache, lz_prefix_init / _free /
   _reset / _match / _prepare / _stats (src/llama_zh.h:781-888,
   src/generate.c:3209-3390) on token ids.  The cache holds a device
   checkpoint of sequence 0's recurrent state and the token prefix it
   covers.  lz_prefix_prepare_tokens is lz_prefix_prepare with the render
   already encoded by the caller: cur = encode(render), pre =
   encode(render[:split]), tail = encode(render[split:]).  It checks that
   the split is token-exact (else the full path: *out_start_pos = 0), that
   the cached prefix is a prefix of cur and that the state was not reset
   since the save (the checkpoint's epoch), restores on a hit, forwards the
   rest of pre, saves the new prefix and returns 0 with *out_start_pos =
   n_pre and *out_reused = the tokens not re-forwarded; generate from there
   with lz_generate_resume(m, s, *out_start_pos, tail, n_tail, ...).  A
   failed forward resets the state and the cache (LZ98_ERR_FORWARD). */
typedef struct LZPrefixCache LZPrefixCache;
int  lz_prefix_init(LZPrefixCache **out, const LZModel *m, char *errbuf, int errlen);
void lz_prefix_free(LZPrefixCache *pc);
void lz_prefix_reset(LZPrefixCache *pc);
int  lz_prefix_match(const LZPrefixCache *pc, const int *pre, int n_pre);
int  lz_prefix_prepare_tokens(LZPrefixCache *pc, const LZModel *m, LZRunState *s, const int *cur, int n_cur,
                              const int *pre, int n_pre, const int *tail, int n_tail, int *out_start_pos,
                              int *out_reused, char *errbuf, int errlen);
void lz_prefix_stats(const LZPrefixCache *pc, long *calls, long *hits, long *tokens_saved, long *mismatch,
                     long *unsplittable);

/* (no counterpart in the reference) Running totals of sequence `seq` over
   its device rounds: rounds, emitted
   tokens (n_accept + 1 per round), accepted drafts, drafted tokens. */
int lz_state_counters(const LZRunState *s, int seq, int *rounds, int *emitted,
                      int *accepted, int *drafted);
/* Measurement hook (no counterpart in the reference): one eager round of
   depth k with CUDA events
   around every int8 GEMV launch.  Returns the summed GEMV device time, their
   algorithmic bytes (weights, scales, activations, outputs), the GEMV count,
   the round's device time and its kernel count. */
int lz_profile_round(LZRunState *s, int k, double *gemv_ms, double *gemv_bytes,
                     int *n_gemv, double *round_ms, int *n_kernels);
/* Measurement hook (no counterpart in the reference), after
   lz_profile_round: the TMA-staged grouped-expert launches of that
   round (event-timed one by one): summed device time, algorithmic bytes
   (every expert's int8 weights and scales) and launch count. */
int lz_profile_experts(const LZRunState *s, double *ms, double *bytes, int *n);
/* Measurement hook (no counterpart in the reference): one eager round of
   depth k with CUDA events around every kernel launch (launched plainly,
   without programmatic overlap): "kernel<TAB>microseconds" lines into buf
   in launch order.  Returns the launch count, or a negative code. */
int lz_profile_launches(LZRunState *s, int k, char *buf, int buflen);
/* Allocation-free logits (no counterpart in the reference): the tied
   lm_head over n final-normed hidden rows (as lz_forward_verify captures
   them), for callers that cannot allocate device memory themselves - a
   process that must not call cudaMalloc, code running inside another
   runtime's memory pool or budget.  hidden (n x hidden_size) and logits
   (n x vocab) are device pointers the caller owns; stream is a
   cudaStream_t (NULL = the legacy default stream).  The quantised rows go
   to a static device array of at most 64 rows x 4096 columns (larger
   requests return LZ98_ERR_SIZE with a message); it is shared by
   every call, so calls that overlap on the GPU race.  The current device
   must be the one lz_open uploaded the model to (else LZ98_ERR_DEVICE).
   The first call on a device resolves the array's device address
   (cudaGetSymbolAddress, once per device even with several calling
   threads) and should come before any stream capture.  Calls no
   cudaMalloc or cudaFree. */
int lz_lm_head_static(const LZModel *m, const float *hidden, int n, float *logits,
                      void *stream, char *errbuf, int errlen);

/* Test hook (no counterpart in the reference): the device primitive that
   computes the sampler's sequential float sums (softmax normaliser,
   cumulative distributions, top-p mass), run on n host values in one
   block.  mode 0: the sequential sum; 1: the first index whose cumulative
   is > target; 2: the first index whose cumulative is >= target.
   *out_value = the sum, or the cumulative at the hit (the total if none);
   *out_hit = the index or -1. */
int lz_debug_seq_sum(const float *vals, int n, int mode, float target, float *out_value,
                     int *out_hit);
/* Test hook: the split sequential sum of squares of the input norms
   (src/ops_norm.c:718, the sum the RMSNorm scale divides) over nrows
   (1-4) host rows of n floats (n a multiple of 512, at most 4096), one
   128-thread group per row; out[r] = row r's sum, which must equal the
   sequential float32 sum of the float32 squares bit for bit. */
int lz_debug_sumsq_split(const float *rows, int nrows, int n, float *out);
/* Test hook: lz_argmax_p1 (src/sampler.c:279-295) of n host values on the
   device - the arg-max and the online-softmax probability the greedy
   p_min compares. */
int lz_debug_argmax_p1(const float *vals, int n, int *out_idx, float *out_p1);
/* Test hook (no counterpart in the reference): a kernel waits on an
   mbarrier that nothing arrives on; its
   bounded wait (about a second, the limit every wait of this library has)
   gives up and reports 2 in *out_err without a fault.  *out_ms: the call's
   duration. */
int lz_debug_wait_timeout(int *out_err, double *out_ms);

/* Test hook (no counterpart in the reference): with `on` nonzero, the
   producer of every TMA-staged launch (the GEMMs and grouped experts of
   rounds with more than 8 token rows) issues nothing for its first
   pipeline stage, and every bounded device wait gives up after limit_ms
   instead of about a second.  The consumers' waits on that stage run out,
   the launch sets the state's error word (no copy is in flight: the
   skipped stage was never issued, every issued one is waited for) and the
   round returns LZ98_ERR_CUDA.  on = 0 restores both.  Acts on the
   current device. */
int lz_debug_inject_wait_timeout(int on, double limit_ms);

/* ---- debug data (src/forward.c:86-124, src/generate.c:226): host
   microseconds spent in capture forwards, verify forwards, draft steps and
   catch-ups, the capture and catch-up call counts, and the rounds that
   rolled the state ring back (n_accept < k_eff, counted by lz_spec_round /
   lz_spec_round_temp).  The direct entry points time themselves; the
   parts of a device round are timed by CUDA events only while
   lz_set_debug_timing(s, 1) is on (the events cut the programmatic-launch
   overlap at their boundaries, so it is off by default). */
extern long long lz_debug_us_verify, lz_debug_us_draft, lz_debug_us_capture, lz_debug_us_catchup;
extern long long lz_debug_n_capture, lz_debug_n_catchup, lz_debug_n_ring_rollback;
int lz_set_debug_timing(LZRunState *s, int enable);

/* ---- recurrent-state checkpoints: replace lz_ckpt_alloc / lz_ckpt_free /
   lz_ckpt_save / lz_ckpt_restore (src/forward.h:1847-1862,
   src/forward_ckpt.c:75-342).  The checkpoint lives in device memory; it
   holds the KDA state planes and scales and the conv history of the
   state's current ring slot (the KV cache is not copied, as in the
   reference), the saved position and the state's epoch.  Restore writes
   ring slot 0 and points the ring there; it refuses an empty checkpoint
   (LZ98_ERR_CKPT_EMPTY), a state reset or reallocated since the save
   (LZ98_ERR_CKPT_STALE) and a shape mismatch (LZ98_ERR_CKPT_SHAPE).  The
   reference signatures act on sequence 0; the _seq forms on any sequence
   of a batched state. */
typedef struct LZStateCkpt LZStateCkpt;
int  lz_ckpt_alloc(LZStateCkpt **out, const LZModel *m, char *errbuf, int errlen);
void lz_ckpt_free(LZStateCkpt *ck);
int  lz_ckpt_save(LZStateCkpt *ck, const LZRunState *s, const LZModel *m, int pos,
                  char *errbuf, int errlen);
int  lz_ckpt_restore(const LZStateCkpt *ck, LZRunState *s, const LZModel *m, int *out_pos,
                     char *errbuf, int errlen);
int  lz_ckpt_save_seq(LZStateCkpt *ck, const LZRunState *s, int seq, int pos, char *errbuf,
                      int errlen);
int  lz_ckpt_restore_seq(const LZStateCkpt *ck, LZRunState *s, int seq, int *out_pos,
                         char *errbuf, int errlen);

/* (no counterpart in the reference) Stream the library launches on
   (cudaStream_t, NULL = a private stream). */
void *lz_state_stream(LZRunState *s);
/* (no counterpart in the reference) Kernels this library launched since
   the state was created. */
long long lz_state_launches(const LZRunState *s);

#ifdef __cplusplus
}
#endif
#endif
