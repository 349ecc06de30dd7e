/* Test infrastructure: the LZSampler fields whose offsets the layout test
   compares between the reference's src/sampler.h and include/lz98_gpu.h. */
#include <stddef.h>
#define LZ98_SAMPLER_FIELDS(X)                                                                 \
    X(vocab_size) X(p.temperature) X(p.temp_think) X(p.think_temp_enabled) X(p.topp) X(p.minp)  \
    X(p.topk) X(p.presence_penalty) X(p.frequency_penalty) X(p.repetition_penalty)             \
    X(p.repeat_last_n) X(p.minp_llamacpp) X(rng_state) X(probindex) X(counts) X(ring) X(cap)   \
    X(head) X(n_win)
#define LZ98_OFF(f) o[n++] = offsetof(LZSampler, f);
#define LZ98_LAYOUT_BODY                          \
    int n = 0;                                    \
    LZ98_SAMPLER_FIELDS(LZ98_OFF)                 \
    o[n++] = sizeof(LZSampler);                   \
    o[n++] = sizeof(LZSampleParams);              \
    o[n++] = sizeof(LZProbIndex);                 \
    return n;
