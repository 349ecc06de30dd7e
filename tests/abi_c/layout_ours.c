/* Test infrastructure: LZSampler offsets under include/lz98_gpu.h alone. */
#include "lz98_gpu.h"
#include "layout.h"
int our_layout(size_t *o) { LZ98_LAYOUT_BODY }
