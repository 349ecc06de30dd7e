/* Test infrastructure: LZSampler offsets under the reference's sampler.h. */
#include "sampler.h"
#include "layout.h"
int ref_layout(size_t *o) { LZ98_LAYOUT_BODY }
