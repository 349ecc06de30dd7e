// Device numerics of the MTP speculative-decoding path, op for op the
// reference engine's float tier (--fixed off, --fastfp off): IEEE binary32,
// round-to-nearest, no fused multiply-add (this translation unit is built
// with -fmad=false), no flush-to-zero, IEEE-rounded division.
// Every helper names the reference file:line whose operation order it keeps.
#pragma once
#include <cstdint>
#include <cfloat>

#define LZ_HD __device__ __forceinline__

namespace lz98 {

constexpr float kLoScale = 256.0f;   // two-plane state, src/ops.h:1922
constexpr float kL2Eps = 1e-6f;      // src/forward.h:23

// src/ops_quant.c:126-135: magic seed, two Newton steps.
LZ_HD float rsqrt_body(float x) {
  float h = __fmul_rn(0.5f, x);
  float y = __uint_as_float(0x5f375a86u - (__float_as_uint(x) >> 1));
  y = __fmul_rn(y, __fsub_rn(1.5f, __fmul_rn(__fmul_rn(h, y), y)));
  y = __fmul_rn(y, __fsub_rn(1.5f, __fmul_rn(__fmul_rn(h, y), y)));
  return y;
}

// 2^(i/32), the reference's own table (src/ops_quant.c:244-253).  Kept in
// global memory and read through the read-only cache: the 32 entries share
// one 128-byte line, so a warp's divergent lookups are one access (constant
// memory would serialise them).
__device__ const float kExpTab32[32] = {
    1.000000000f, 1.021897149f, 1.044273782f, 1.067140401f,
    1.090507733f, 1.114386743f, 1.138788635f, 1.163724859f,
    1.189207115f, 1.215247360f, 1.241857812f, 1.269050957f,
    1.296839555f, 1.325236643f, 1.354255547f, 1.383909882f,
    1.414213562f, 1.445180807f, 1.476826146f, 1.509164428f,
    1.542210825f, 1.575980845f, 1.610490332f, 1.645755478f,
    1.681792831f, 1.718619298f, 1.756252160f, 1.794709075f,
    1.834008086f, 1.874167634f, 1.915206561f, 1.957144124f,
};

// src/ops_quant.c:300-349: exponent/32-step split by the 1.5*2^23 magic
// add, quadratic in w = 1 + r/32, table times polynomial times 2^n.
LZ_HD float exp_body(float x) {
  if (x > 88.0f) return FLT_MAX;
  if (x < -87.3f) return 0.0f;
  const float log2e32 = 1.44269504f * 32.0f;
  float y32 = __fmul_rn(x, log2e32);
  float u = __fadd_rn(__fsub_rn(y32, 0.5f), 12582912.0f);
  int t = (__float_as_int(u) & 0x007FFFFF) - 0x00400000;
  int n = t >> 5;
  int idx = t & 31;
  float r = __fsub_rn(y32, (float)t);
  float w = __fadd_rn(1.0f, __fmul_rn(r, 0.03125f));
  float p2n = __int_as_float((n + 127) << 23);
  float c = __fadd_rn(__fmul_rn(__fadd_rn(__fmul_rn(0.242844437f, w), 0.207425515f), w), 0.549730133f);
  return __fmul_rn(p2n, __fmul_rn(__ldg(kExpTab32 + idx), c));
}

// src/ops_quant.c:1836-1842 (float arm).
LZ_HD float sigmoid(float x) {
  if (x >= 0.0f) {
    float z = exp_body(-x);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
  }
  float z = exp_body(x);
  return __fdiv_rn(z, __fadd_rn(1.0f, z));
}

LZ_HD float silu(float x) { return __fmul_rn(x, sigmoid(x)); }

// src/ops_quant.h:181-186 under round-to-nearest: half-to-even rounding
// of |v| < 2^22 through the magic add.
LZ_HD int q8_round(float v) {
  return (__float_as_int(__fadd_rn(v, 12582912.0f)) & 0x007FFFFF) - 0x00400000;
}
LZ_HD int q8_clamp(int q) { return q > 127 ? 127 : (q < -127 ? -127 : q); }

// src/ops_quant.c:1633-1666 given the group's magnitude bits.
LZ_HD void q8_scale_from_amax(uint32_t am_bits, float* sg, float* inv) {
  float amax = __uint_as_float(am_bits);
  if (amax > 0.0f) {
    *sg = __fmul_rn(amax, 1.0f / 127.0f);
    *inv = __fdiv_rn(127.0f, amax);
    if (*sg < 1.0e-30f) { *sg = 1.0f; *inv = 0.0f; }
  } else {
    *sg = 1.0f;
    *inv = 0.0f;
  }
}

LZ_HD uint32_t abs_bits(float x) { return __float_as_uint(x) & 0x7FFFFFFFu; }

// Max over the 32 lanes of a warp (every lane gets it): one redux.sync
// (~22 cycles here, against ~130 for five shuffle steps).
LZ_HD uint32_t warp_max_u32(uint32_t v) { return __reduce_max_sync(0xffffffffu, v); }

// Max of a 64-bit value over the 32 lanes (every lane gets it): the max of
// the high words, then of the low words among the lanes holding that high
// word - two redux.sync instead of five two-word shuffle steps.
LZ_HD unsigned long long warp_max_u64(unsigned long long v) {
  const uint32_t hi = (uint32_t)(v >> 32), mh = __reduce_max_sync(0xffffffffu, hi);
  const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? (uint32_t)v : 0u);
  return ((unsigned long long)mh << 32) | ml;
}

// One 32-element activation group held one element per lane: the
// reference quantiser (src/ops_quant.c:2152-2282). Returns the code; the
// group scale is written by lane 0 when `scale_out` is non-null.
LZ_HD int8_t warp_quant32(float x, float* scale_out) {
  uint32_t am = warp_max_u32(abs_bits(x));
  float sg, inv;
  q8_scale_from_amax(am, &sg, &inv);
  if (scale_out && (threadIdx.x & 31) == 0) *scale_out = sg;
  return (int8_t)q8_clamp(q8_round(__fmul_rn(x, inv)));
}

// Total-order key of src/sampler.c:224: larger float -> larger key.
LZ_HD uint32_t fkey(float f) {
  uint32_t u = __float_as_uint(f);
  return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
}

// xorshift64*, top 24 bits over 2^24 (src/sampler.c:185-203).
LZ_HD float random_f32(unsigned long long* st) {
  unsigned long long x = *st;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  *st = x;
  unsigned int r = (unsigned int)((x * 0x2545F4914F6CDD1DULL) >> 32);
  return __fdiv_rn((float)(r >> 8), 16777216.0f);
}

// Programmatic dependent launch (sm_90+): let the next kernel of the
// stream start its independent prologue now, and wait here until every
// prerequisite grid has completed and its writes are visible.  Both are
// no-ops for a kernel launched without the programmatic attribute.
LZ_HD void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
LZ_HD void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Thread-block clusters: this CTA's rank in its cluster, the cluster-wide
// barrier (every thread of every CTA of the cluster; release / acquire, so
// shared-memory writes before it are visible to the peers after it), and a
// float written to / read from the same shared-memory variable of a peer
// CTA.
LZ_HD uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
LZ_HD void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
LZ_HD void st_peer_f32(float* local, uint32_t peer, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"((uint32_t)__cvta_generic_to_shared(local)),
               "r"(peer));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}
LZ_HD float ld_peer_f32(const float* local, uint32_t peer) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"((uint32_t)__cvta_generic_to_shared(local)),
               "r"(peer));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// ------------------------------------------------ TMA, mbarriers, ldmatrix

LZ_HD uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

LZ_HD void mbar_init(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// make barrier initialisation visible to the async (TMA) proxy
LZ_HD void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// Order the consumers' generic-proxy reads of a pipeline stage (released to
// the producer through the stage's empty mbarrier) before the TMA writes
// (async proxy) that refill it.  Without it a refill can land while a
// consumer's shared-memory reads of the previous contents are still
// outstanding: a rare, timing-dependent wrong product (observed as
// run-to-run differences of batch-32 temperature rounds under programmatic
// dependent launch).
LZ_HD void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
LZ_HD void mbar_expect_tx(uint32_t bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
LZ_HD void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
LZ_HD bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
LZ_HD unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Limit of every bounded device wait (about a second), and a test switch
// that makes the producer of every TMA-staged launch issue nothing for its
// first pipeline stage; both set only by lz_debug_inject_wait_timeout.
__device__ unsigned long long g_wait_limit_ns = 1000000000ull;
__device__ int g_dbg_skip_stage = 0;

// Wait until the phase of parity `parity` of the barrier has completed,
// giving up after g_wait_limit_ns (returns false): no wait in this library
// can spin for ever.
LZ_HD bool mbar_wait(uint32_t bar, uint32_t parity) {
#pragma unroll 1
  for (int i = 0; i < 256; i++)
    if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns(), lim = g_wait_limit_ns;
#pragma unroll 1
  while (!mbar_try(bar, parity))
    if (global_ns() - t0 > lim) return false;
  return true;
}
// 2-D tiled TMA load of the box at (x, y) (x in elements of the innermost
// dimension) into shared memory, completing on the barrier.
LZ_HD void tma_load_2d(uint32_t dst, const void* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
LZ_HD void ldsm_x4(uint32_t addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
LZ_HD void ldsm_x2(uint32_t addr, unsigned& r0, unsigned& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// Ask L2 to fetch [p, p + bytes) from HBM without waiting (bulk prefetch,
// sm_90+).  p must be 16-byte aligned; the range is cut down to whole
// 16-byte units so that it never reaches past the caller's buffer.
LZ_HD void prefetch_l2(const void* p, size_t bytes) {
  const char* c = static_cast<const char*>(p);
  bytes &= ~(size_t)15;
  while (bytes) {
    const unsigned n = bytes > 65536 ? 65536u : (unsigned)bytes;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
    c += n;
    bytes -= n;
  }
}

}  // namespace lz98
