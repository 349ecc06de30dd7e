// Temperature sampling of the speculative round on the device: the draft
// distribution q and its sample (lz_sample_temp_q), the target distribution
// p with top-p (lz_target_dist), the coupled acceptance with residual
// resampling (lz_spec_accept_temp) and the top-p sample of a first anchor
// (sample_ex).  Every float operation keeps the reference's order:
// sequential index-order sums and cumulative sums (src/ops_norm.c:903-985,
// src/sampler.c:526-745, src/generate.c:264-349).
//
// The sequential sums are the critical path.  They run on one thread of a
// 1024-thread block while the other 31 warps compute the next values into
// shared memory, and the thread writes the running sum back in place so the
// block can find the first position whose cumulative passes a threshold in
// parallel (a cumulative sum of non-negative values is non-decreasing, so
// "threshold reached" is monotone along the array).
#pragma once
#include <climits>
#include "lz98_kernels.cuh"

namespace lz98 {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kChainStage = 2048;      // values per staged chunk
constexpr int kSortChunk = 8192;       // bitonic stages below this run in shared memory
constexpr float kTempFloor = 1e-3f;    // LZ_TEMP_FLOOR, src/sampler.h:130

// Dynamic shared memory of every sampling kernel (the chain's three stage
// buffers and the sort chunk share it).
constexpr size_t kSampSmem = (size_t)kSortChunk * sizeof(float);
static_assert(3 * kChainStage <= kSortChunk, "stage buffers must fit the sort chunk");

struct SampShared {
  float red_f[kSampWarps];
  uint32_t red_u[kSampWarps];
  int red_i[kSampWarps];
  float acc;
  int hit;
  int carry;
  int bcast_i[4];
  float bcast_f[4];
};

LZ_HD float key_float(uint32_t k) {        // inverse of fkey
  return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

LZ_HD uint32_t block_max_u32(uint32_t v, SampShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max_u32(v);
  __syncthreads();
  if (lane == 0) sh.red_u[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kSampWarps ? sh.red_u[lane] : 0u;
    w = warp_max_u32(w);
    if (lane == 0) sh.red_u[0] = w;
  }
  __syncthreads();
  return sh.red_u[0];
}

LZ_HD int block_sum_i(int v, SampShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh.red_i[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kSampWarps ? sh.red_i[lane] : 0;
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0) sh.red_i[0] = w;
  }
  __syncthreads();
  return sh.red_i[0];
}

LZ_HD int block_max_i(int v, SampShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) sh.red_i[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kSampWarps ? sh.red_i[lane] : INT_MIN;
    for (int o = 16; o > 0; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) sh.red_i[0] = w;
  }
  __syncthreads();
  return sh.red_i[0];
}

enum ChainMode { kChainSum = 0, kChainFindLt = 1, kChainFindGe = 2 };

// Sequential float sum acc = ((0 + v(0)) + v(1)) + ... over j < n (values
// must be >= 0 for the find modes).  kChainSum returns the total.  The find
// modes stop at the first j whose cumulative c satisfies target < c
// (kChainFindLt) or c >= target (kChainFindGe): *hit = j and the return
// value is c; with no such j, *hit = -1 and the total is returned.
// Called by every thread of the block; `stage` holds 3 * kChainStage floats.
template <int MODE, class F>
__device__ float block_chain(F val, int n, float target, float* stage, SampShared& sh, int* hit) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nch = (n + kChainStage - 1) / kChainStage;
  for (int t = tid; t < min(kChainStage, n); t += kSampThreads) stage[t] = val(t);
  if (tid == 0) { sh.hit = -1; sh.acc = 0.0f; }
  __syncthreads();
  float acc = 0.0f;
  int found = -1;
  for (int c = 0; c <= nch && found < 0; c++) {
    if (tid == 0 && c < nch) {
      float* b = stage + (c % 3) * kChainStage;
      const int len = min(kChainStage, n - c * kChainStage);
      int t = 0;
      for (; t + 4 <= len; t += 4) {
        float4 v4 = *reinterpret_cast<float4*>(b + t);
        v4.x = acc = __fadd_rn(acc, v4.x);
        v4.y = acc = __fadd_rn(acc, v4.y);
        v4.z = acc = __fadd_rn(acc, v4.z);
        v4.w = acc = __fadd_rn(acc, v4.w);
        if (MODE != kChainSum) *reinterpret_cast<float4*>(b + t) = v4;
      }
      for (; t < len; t++) {
        acc = __fadd_rn(acc, b[t]);
        if (MODE != kChainSum) b[t] = acc;
      }
    } else if (warp > 0) {
      // the previous chunk's cumulatives: first position meeting the target
      if (MODE != kChainSum && c >= 1) {
        const float* b = stage + ((c - 1) % 3) * kChainStage;
        const int base = (c - 1) * kChainStage, len = min(kChainStage, n - base);
        for (int t = tid - 32; t < len; t += kSampThreads - 32) {
          const float cu = b[t];
          const bool ok = MODE == kChainFindLt ? (target < cu) : (cu >= target);
          const bool prev = t > 0 && (MODE == kChainFindLt ? (target < b[t - 1]) : (b[t - 1] >= target));
          if (ok && !prev) { sh.hit = base + t; sh.acc = cu; }
        }
      }
      if (c + 1 < nch) {
        float* b = stage + ((c + 1) % 3) * kChainStage;
        const int base = (c + 1) * kChainStage, len = min(kChainStage, n - base);
        for (int t = tid - 32; t < len; t += kSampThreads - 32) b[t] = val(base + t);
      }
    }
    __syncthreads();
    found = sh.hit;
  }
  if (found < 0) {
    if (tid == 0) sh.acc = acc;
    __syncthreads();
  }
  const float r = sh.acc;
  if (hit) *hit = found;
  __syncthreads();
  return r;
}

// Numerically the reference softmax of logits * inv_t (src/ops_norm.c:903-985
// after src/sampler.c:736-745 scaling): max by order key, exp(x - max) by the
// reference's exp body, sequential sum, times 1/sum.  Writes probabilities
// to out.  Returns nothing; every thread must call.
__device__ void block_softmax(const float* __restrict__ lg, int n, float inv_t, float* out, float* stage,
                              SampShared& sh) {
  uint32_t best = 0;
  for (int j = threadIdx.x; j < n; j += kSampThreads) {
    const uint32_t k = fkey(__fmul_rn(__ldcg(lg + j), inv_t));
    best = k > best ? k : best;
  }
  const float mx = key_float(block_max_u32(best, sh));
  auto ev = [&](int j) { return exp_body(__fsub_rn(__fmul_rn(__ldcg(lg + j), inv_t), mx)); };
  const float sum = block_chain<kChainSum>(ev, n, 0.0f, stage, sh, nullptr);
  const float invs = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
  for (int j = threadIdx.x; j < n; j += kSampThreads) out[j] = __fmul_rn(ev(j), invs);
  __syncthreads();
}

// First index of the maximum by order key (src/sampler.c:224-240).
__device__ int block_argmax(const float* v, int n, SampShared& sh) {
  unsigned long long best = 0ull;
  for (int j = threadIdx.x; j < n; j += kSampThreads) {
    const unsigned long long k = ((unsigned long long)fkey(__ldcg(v + j)) << 32) | (uint32_t)~(uint32_t)j;
    best = k > best ? k : best;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, best, o);
    best = w > best ? w : best;
  }
  __shared__ unsigned long long red[kSampWarps];
  __syncthreads();
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kSampWarps; w++) b = red[w] > b ? red[w] : b;
    red[0] = b;
  }
  __syncthreads();
  const int r = (int)~(uint32_t)(red[0] & 0xffffffffull);
  __syncthreads();
  return r;
}

// Descending bitonic sort of a[0..N), N a power of two >= 2, by one block:
// stages whose partner distance is below the chunk run in shared memory.
__device__ void block_sort_desc(float* a, int N, float* sh) {
  const int S = min(N, kSortChunk);
  auto cx = [](float* v, int i, int l, bool desc) {
    const float x = v[i], y = v[l];
    if (desc ? (x < y) : (x > y)) { v[i] = y; v[l] = x; }
  };
  // phase 1: sort every chunk (direction alternating with the chunk's place
  // in the global network)
  for (int c0 = 0; c0 < N; c0 += S) {
    for (int t = threadIdx.x; t < S; t += kSampThreads) sh[t] = a[c0 + t];
    __syncthreads();
    for (int k = 2; k <= S; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int t = threadIdx.x; t < S / 2; t += kSampThreads) {
          const int i = (t / j) * 2 * j + (t % j);
          cx(sh, i, i + j, ((c0 + i) & k) == 0);
        }
        __syncthreads();
      }
    for (int t = threadIdx.x; t < S; t += kSampThreads) a[c0 + t] = sh[t];
    __syncthreads();
  }
  // merges across chunks
  for (int k = 2 * S; k <= N; k <<= 1) {
    for (int j = k >> 1; j >= S; j >>= 1) {
      for (int t = threadIdx.x; t < N / 2; t += kSampThreads) {
        const int i = (t / j) * 2 * j + (t % j);
        cx(a, i, i + j, (i & k) == 0);
      }
      __syncthreads();
    }
    for (int c0 = 0; c0 < N; c0 += S) {
      for (int t = threadIdx.x; t < S; t += kSampThreads) sh[t] = a[c0 + t];
      __syncthreads();
      for (int j = S >> 1; j > 0; j >>= 1) {
        for (int t = threadIdx.x; t < S / 2; t += kSampThreads) {
          const int i = (t / j) * 2 * j + (t % j);
          cx(sh, i, i + j, ((c0 + i) & k) == 0);
        }
        __syncthreads();
      }
      for (int t = threadIdx.x; t < S; t += kSampThreads) a[c0 + t] = sh[t];
      __syncthreads();
    }
  }
}

// The r-th (0-based) index j in ascending order with p[j] == v, by tiles of
// the block with a running carry; -1 if there is none.
__device__ int block_nth_equal(const float* p, int n, float v, int r, SampShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) { sh.carry = 0; sh.bcast_i[0] = -1; }
  __syncthreads();
  for (int j0 = 0; j0 < n; j0 += kSampThreads) {
    const int j = j0 + threadIdx.x;
    const bool eq = j < n && p[j] == v;
    const unsigned m = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) sh.red_i[warp] = __popc(m);
    __syncthreads();
    int before = sh.carry;
    for (int w = 0; w < warp; w++) before += sh.red_i[w];
    before += __popc(m & ((1u << lane) - 1u));
    if (eq && before == r) sh.bcast_i[0] = j;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < kSampWarps; w++) tot += sh.red_i[w];
      sh.carry += tot;
    }
    __syncthreads();
    if (sh.bcast_i[0] >= 0) break;
  }
  const int res = sh.bcast_i[0];
  __syncthreads();
  return res;
}

// Result of the top-p candidate selection (src/sampler.c:526-652 with
// topk = 0, minp = 0): candidates p >= cut sorted descending (ties by
// ascending index), cut at the first cumulative >= topp.
struct Nucleus {
  int n0;          // candidates
  int last;        // last kept position in sorted order (-1: none)
  float mass;      // cumulative at the cut
};

// p holds the softmax probabilities (length n); sorted is scratch of
// npow2 floats; returns the nucleus.
__device__ Nucleus block_nucleus(const float* p, int n, float topp, float* sorted, int npow2, float* stage,
                                 SampShared& sh) {
  const float cut = n > 1 ? __fdiv_rn(__fsub_rn(1.0f, topp), (float)(n - 1)) : 0.0f;
  int cnt = 0;
  for (int j = threadIdx.x; j < npow2; j += kSampThreads) {
    const float v = j < n ? p[j] : -1.0f;
    const bool c = j < n && v >= cut;
    sorted[j] = c ? v : -1.0f;
    cnt += c;
  }
  Nucleus nu;
  nu.n0 = block_sum_i(cnt, sh);
  nu.last = -1;
  nu.mass = 0.0f;
  if (nu.n0 <= 0) return nu;
  block_sort_desc(sorted, npow2, stage);
  int hit;
  auto sv = [&](int j) { return sorted[j]; };
  const float limit = __fmul_rn(topp, 1.0f);
  const float c = block_chain<kChainFindGe>(sv, nu.n0, limit, stage, sh, &hit);
  nu.last = hit >= 0 ? hit : nu.n0 - 1;
  nu.mass = c;
  return nu;
}

// Number of sorted positions before the first one equal to sorted[pos].
__device__ int block_first_pos(const float* sorted, int pos, SampShared& sh) {
  const float v = sorted[pos];
  int c = 0;
  for (int j = threadIdx.x; j < pos; j += kSampThreads) c += sorted[j] > v;
  return block_sum_i(c, sh);
}

// lz_target_dist (src/sampler.c:682-714): p row in place; sorted is
// npow2 floats of scratch.
__device__ void block_target_dist(const float* lg, int n, float temp, float topp, float* p, float* sorted,
                                  int npow2, float* stage, SampShared& sh) {
  const float inv_t = __fdiv_rn(1.0f, temp);
  block_softmax(lg, n, inv_t, p, stage, sh);
  if (topp <= 0.0f || topp >= 1.0f) return;
  const Nucleus nu = block_nucleus(p, n, topp, sorted, npow2, stage, sh);
  if (nu.last < 0) {
    const int am = block_argmax(p, n, sh);
    for (int j = threadIdx.x; j < n; j += kSampThreads) p[j] = j == am ? 1.0f : 0.0f;
    __syncthreads();
    return;
  }
  // kept: every p > v_last, and the first `need` (by index) of p == v_last
  const float vl = sorted[nu.last];
  const int need = nu.last + 1 - block_first_pos(sorted, nu.last, sh);
  if (threadIdx.x == 0) sh.carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int j0 = 0; j0 < n; j0 += kSampThreads) {
    const int j = j0 + threadIdx.x;
    const float v = j < n ? p[j] : 0.0f;
    const bool eq = j < n && v == vl;
    const unsigned m = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) sh.red_i[warp] = __popc(m);
    __syncthreads();
    int before = sh.carry;
    for (int w = 0; w < warp; w++) before += sh.red_i[w];
    before += __popc(m & ((1u << lane) - 1u));
    if (j < n) {
      const bool keep = v > vl || (eq && before < need);
      p[j] = keep ? __fdiv_rn(v, nu.mass) : 0.0f;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < kSampWarps; w++) tot += sh.red_i[w];
      sh.carry += tot;
    }
    __syncthreads();
  }
}

// sample_ex with identity penalties (src/sampler.c:794-901): the coin is
// drawn first; top-p sample from the sorted nucleus.  p and sorted are
// scratch rows (n and npow2 floats).  Thread 0 owns *rng.
__device__ int block_sample_ex(const float* lg, int n, float temp, float topp, unsigned long long* rng, float* p,
                               float* sorted, int npow2, float* stage, SampShared& sh) {
  if (!(temp > kTempFloor)) return block_argmax(lg, n, sh);
  if (threadIdx.x == 0) sh.bcast_f[0] = random_f32(rng);
  __syncthreads();
  const float coin = sh.bcast_f[0];
  const float inv_t = __fdiv_rn(1.0f, temp);
  block_softmax(lg, n, inv_t, p, stage, sh);
  int hit;
  if (topp <= 0.0f || topp >= 1.0f) {
    auto pv = [&](int j) { return p[j]; };
    block_chain<kChainFindLt>(pv, n, coin, stage, sh, &hit);
    return hit >= 0 ? hit : n - 1;
  }
  const Nucleus nu = block_nucleus(p, n, topp, sorted, npow2, stage, sh);
  if (nu.last < 0) return block_argmax(p, n, sh);
  const float r = __fmul_rn(coin, nu.mass);
  auto sv = [&](int j) { return sorted[j]; };
  block_chain<kChainFindLt>(sv, nu.last + 1, r, stage, sh, &hit);
  const int pos = hit >= 0 ? hit : nu.last;
  const int first = block_first_pos(sorted, pos, sh);
  return block_nth_equal(p, n, sorted[pos], pos - first, sh);
}

// ------------------------------------------------------------ round kernels

// Draft step i of every sequence in temperature mode (src/generate.c:1234-1300
// with lz_sample_temp_q, src/sampler.c:736-745): q = softmax(logits / T)
// kept for the acceptance, coin from the sequence's generator, first index
// whose cumulative q exceeds the coin (the last index if none).
__global__ void __launch_bounds__(kSampThreads) temp_draft_kernel(const float* __restrict__ logits, int V,
                                                                  SeqRound* sr, int i, int k, int kmax,
                                                                  float* qbuf) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  const int b = blockIdx.x;
  SeqRound& s = sr[b];
  float* q = qbuf + ((size_t)b * kmax + i) * V;
  block_softmax(logits + (size_t)b * V, V, __fdiv_rn(1.0f, s.temp), q, stage, sh);
  if (threadIdx.x == 0) sh.bcast_f[0] = random_f32(&s.rng);
  __syncthreads();
  const float coin = sh.bcast_f[0];
  int hit;
  auto qv = [&](int j) { return q[j]; };
  block_chain<kChainFindLt>(qv, V, coin, stage, sh, &hit);
  if (threadIdx.x == 0) {
    s.draft[i] = hit >= 0 ? hit : V - 1;
    s.k = k;
  }
}

// Target distributions of every verify row (lz_target_dist with the
// sequence's temperature and top-p), one block per row b * (k + 1) + j.
__global__ void __launch_bounds__(kSampThreads) temp_target_kernel(const float* __restrict__ logits, int V,
                                                                   const SeqRound* sr, int k, float* pbuf,
                                                                   float* sortbuf, int npow2) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  const int row = blockIdx.x, b = row / (k + 1);
  block_target_dist(logits + (size_t)row * V, V, sr[b].temp, sr[b].topp, pbuf + (size_t)row * V,
                    sortbuf + (size_t)row * npow2, npow2, stage, sh);
}

// Coupled acceptance of a temperature round (src/generate.c:1300-1377 with
// lz_spec_accept_temp, src/generate.c:264-349): for each draft x_i,
// u < min(1, p(x_i)/q(x_i)) accepts; the first rejection resamples from the
// residual max(0, p - q) and ends the round; with every draft accepted the
// bonus token is sampled from the last target row.  Then the bookkeeping
// and the chain reseed of the greedy round.
__global__ void __launch_bounds__(kSampThreads) temp_accept_kernel(
    SeqRound* sr, int k, int kmax, const float* __restrict__ pbuf, const float* __restrict__ qbuf, int V,
    const float* __restrict__ vhid, int d, float* chain, int depth, int seq_len, MtpRow* catch_rows,
    int* catch_tok, int* catch_hidx) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  const int b = blockIdx.x;
  SeqRound& s = sr[b];
  const int row0 = b * (k + 1);
  int n_accept = k;
  for (int i = 0; i < k; i++) {
    const float* p = pbuf + (size_t)(row0 + i) * V;
    const float* q = qbuf + ((size_t)b * kmax + i) * V;
    if (threadIdx.x == 0) {
      const float u = random_f32(&s.rng);
      const int x = s.draft[i];
      const float qx = q[x];
      float ratio = 0.0f;
      if (qx > 0.0f) {
        ratio = __fdiv_rn(p[x], qx);
        if (ratio > 1.0f) ratio = 1.0f;
      }
      sh.bcast_i[1] = u < ratio;
      if (u < ratio) s.out[i] = x;
    }
    __syncthreads();
    const bool acc = sh.bcast_i[1];
    __syncthreads();
    if (acc) continue;
    // residual max(0, p - q): sequential total, then the sample
    auto dv = [&](int j) {
      const float dd = __fsub_rn(p[j], q[j]);
      return dd > 0.0f ? dd : 0.0f;
    };
    const float total = block_chain<kChainSum>(dv, V, 0.0f, stage, sh, nullptr);
    int lp = -1;
    for (int j = threadIdx.x; j < V; j += kSampThreads)
      if (__fsub_rn(p[j], q[j]) > 0.0f) lp = j;
    const int last_pos = block_max_i(lp, sh);
    int tok;
    if (total <= 0.0f) {
      tok = block_argmax(p, V, sh);
    } else {
      if (threadIdx.x == 0) sh.bcast_f[1] = __fmul_rn(random_f32(&s.rng), total);
      __syncthreads();
      const float coin = sh.bcast_f[1];
      int hit;
      block_chain<kChainFindLt>(dv, V, coin, stage, sh, &hit);
      tok = hit >= 0 ? hit : last_pos;
    }
    if (threadIdx.x == 0) s.out[i] = tok;
    n_accept = i;
    break;
  }
  if (n_accept == k) {
    const float* p = pbuf + (size_t)(row0 + k) * V;
    if (threadIdx.x == 0) sh.bcast_f[2] = random_f32(&s.rng);
    __syncthreads();
    const float coin = sh.bcast_f[2];
    int hit;
    auto pv = [&](int j) { return p[j]; };
    block_chain<kChainFindLt>(pv, V, coin, stage, sh, &hit);
    if (threadIdx.x == 0) s.out[k] = hit >= 0 ? hit : V - 1;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    round_bookkeeping(s, b, n_accept, k, k, row0, depth, seq_len, catch_rows, catch_tok, catch_hidx);
  for (int t = threadIdx.x; t < d; t += kSampThreads)
    chain[(size_t)b * d + t] = vhid[(size_t)(row0 + n_accept) * d + t];
}

// One token from one logits row with the sequence's sampler (sample_ex,
// src/sampler.c:794-901; arg-max when the temperature is at the floor).
__global__ void __launch_bounds__(kSampThreads) sample_row_kernel(const float* __restrict__ logits, int V,
                                                                  SeqRound* sr, int seq, float* p, float* sorted,
                                                                  int npow2, int* out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  SeqRound& s = sr[seq];
  const int tok = block_sample_ex(logits, V, s.temp, s.topp, &s.rng, p, sorted, npow2, stage, sh);
  if (threadIdx.x == 0) *out = tok;
}

}  // namespace lz98
