// Temperature sampling of the speculative round on the device: the draft
// distribution q and its sample (lz_sample_temp_q), the target distribution
// p with top-p (lz_target_dist), the coupled acceptance with residual
// resampling (lz_spec_accept_temp) and the top-p sample of a first anchor
// (sample_ex).  Every float operation keeps the reference's order:
// sequential index-order sums and cumulative sums (src/ops_norm.c:903-985,
// src/sampler.c:526-745, src/generate.c:264-349).
//
// The sequential sums are the critical path.  block_chain computes them
// exactly but in parallel (binade segments with integer ulp prefix sums),
// see its comment.
#pragma once
#include <climits>
#include "lz98_kernels.cuh"

namespace lz98 {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kSortChunk = 8192;       // bitonic stages below this run in shared memory
constexpr float kTempFloor = 1e-3f;    // LZ_TEMP_FLOOR, src/sampler.h:130

// Dynamic shared memory of every sampling kernel (the chain's three stage
// buffers and the sort chunk share it).
constexpr size_t kSampSmem = (size_t)kSortChunk * sizeof(float);
static_assert(1024 <= kSortChunk, "the chain's head must fit the stage");

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

// ---------------------------------------------------------------------------
// Exact sequential float sums, computed in parallel.
//
// acc_j = fl(acc_{j-1} + v_j) (round to nearest even, v_j >= 0 finite).
// While the running sum s stays in one binade its grid is u = ulp(s), and
// fl(s + v) = s + u * rne(v / u): the rounding of each addend does not
// depend on s, except at an exact tie (v / u ending in .5, where the even
// rule looks at s).  So inside a segment the running sum is s/u plus an
// integer prefix sum of per-addend ulp counts.  A segment ends at the first
// addend that ties or whose rounded prefix reaches the next binade (2^24
// ulps); that addend is added with a real fadd and a new segment starts
// from the exact result.  Every cumulative equals the sequential one bit
// for bit (zeros keep s at 0; the first non-zero addend after them is
// taken exactly).
//
// Values are decomposed as v = M * 2^(E - 150) with E = max(biased
// exponent, 1), which covers subnormals with the same formulas.

LZ_HD void fdecomp(float x, int& E, uint32_t& M) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t e = b >> 23;
  M = (b & 0x7FFFFFu) | (e ? 0x800000u : 0u);
  E = e ? (int)e : 1;
}

// s = m * 2^(E - 150) for m < 2^24 (m < 2^23 only when E == 1)
LZ_HD float frecon(int E, unsigned long long m) {
  return m >= 0x800000ull ? __uint_as_float(((uint32_t)E << 23) | ((uint32_t)m & 0x7FFFFFu))
                          : __uint_as_float((uint32_t)m);
}

// ulps of v = Mj * 2^(Ej - 150) on the grid of exponent Es, rounded to
// nearest; tie flags an exact half.
LZ_HD unsigned long long fulps(int Ej, uint32_t Mj, int Es, bool& tie) {
  tie = false;
  if (Mj == 0u) return 0ull;
  const int sh = Ej - Es;
  if (sh >= 0) return sh >= 7 ? (1ull << 30) : (unsigned long long)(Mj << sh);
  const int r = -sh;
  if (r >= 25) return 0ull;
  const uint32_t q = Mj >> r, rem = Mj & ((1u << r) - 1u), half = 1u << (r - 1);
  tie = rem == half;
  return q + (rem > half ? 1u : 0u);
}

template <int MODE>
LZ_HD bool chain_cond(float c, float target) {
  return MODE == kChainFindLt ? (target < c) : (MODE == kChainFindGe ? (c >= target) : false);
}

constexpr int kChainHead = 1024;      // leading values summed serially
constexpr int kChainPer = 8;          // values per thread per window
constexpr int kChainWin = kChainPer * kSampThreads;

struct ChainShared {
  unsigned long long wt[kSampWarps];  // warp totals, then exclusive offsets
  int wstop[kSampWarps], wfind[kSampWarps];
  int S, F;
  float sum;
  int hit;
};

LZ_HD unsigned long long warp_incl_scan_u64(unsigned long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long w = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += w;
  }
  return v;
}

// Block-wide minima of two ints (warp 0 finishes; two barriers).
LZ_HD void block_min2(int a, int b, ChainShared& cs, int& A, int& B) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = __reduce_min_sync(0xffffffffu, a);
  b = __reduce_min_sync(0xffffffffu, b);
  if (lane == 0) { cs.wstop[warp] = a; cs.wfind[warp] = b; }
  __syncthreads();
  if (warp == 0) {
    const int x = __reduce_min_sync(0xffffffffu, cs.wstop[lane]);
    const int y = __reduce_min_sync(0xffffffffu, cs.wfind[lane]);
    if (lane == 0) { cs.S = x; cs.F = y; }
  }
  __syncthreads();
  A = cs.S;
  B = cs.F;
}

// Sum (kChainSum) or first cumulative meeting the target (find modes) of
// v(0..n-1) in sequential float order.  The find modes stop at the first j
// whose cumulative c satisfies target < c (kChainFindLt) or c >= target
// (kChainFindGe): *hit = j and c is returned; with no such j, *hit = -1 and
// the total is returned.  Every thread of the block calls it; `stage` holds
// kChainHead floats.
template <int MODE, class F>
__device__ float block_chain(F val, int n, float target, float* stage, SampShared& sh, int* hit) {
  __shared__ ChainShared cs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // serial head: crossings are dense while the sum is small
  const int nh = min(n, kChainHead);
  for (int t = tid; t < nh; t += kSampThreads) stage[t] = val(t);
  __syncthreads();
  if (tid == 0) {
    float acc = 0.0f;
    int h = -1;
    for (int t = 0; t < nh; t++) {
      acc = __fadd_rn(acc, stage[t]);
      if (MODE != kChainSum && chain_cond<MODE>(acc, target)) { h = t; break; }
    }
    cs.sum = acc;
    cs.hit = h;
  }
  __syncthreads();
  float s = cs.sum;
  int found = cs.hit;
  for (int w0 = nh; w0 < n && found < 0; w0 += kChainWin) {
    const int j0 = w0 + tid * kChainPer;
    const int wend = min(n, w0 + kChainWin);
    float v[kChainPer];
    int ve[kChainPer];
    uint32_t vm[kChainPer];
#pragma unroll
    for (int k = 0; k < kChainPer; k++) {
      v[k] = j0 + k < wend ? val(j0 + k) : 0.0f;
      fdecomp(v[k], ve[k], vm[k]);
    }
    int cur = w0;                      // first index of the open segment
    while (cur < wend && found < 0) {
      if (s == 0.0f) {
        // the sum stays 0 up to the first non-zero value, taken exactly
        if (MODE != kChainSum && chain_cond<MODE>(0.0f, target)) { found = cur; break; }
        int fz = INT_MAX;
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k >= cur && j0 + k < wend && v[k] > 0.0f) fz = min(fz, j0 + k);
        int z, unused;
        block_min2(fz, INT_MAX, cs, z, unused);
        if (z == INT_MAX) { cur = wend; break; }
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == z) cs.sum = v[k];
        __syncthreads();
        s = cs.sum;
        __syncthreads();
        if (MODE != kChainSum && chain_cond<MODE>(s, target)) { found = z; break; }
        cur = z + 1;
        continue;
      }
      int Es;
      uint32_t Ms;
      fdecomp(s, Es, Ms);
      unsigned long long pre[kChainPer], nu[kChainPer];
      bool tie[kChainPer];
      unsigned long long run = 0ull;
#pragma unroll
      for (int k = 0; k < kChainPer; k++) {
        const bool live = j0 + k >= cur && j0 + k < wend;
        nu[k] = live ? fulps(ve[k], vm[k], Es, tie[k]) : 0ull;
        tie[k] = live && tie[k];
        run += nu[k];
        pre[k] = run;
      }
      // block exclusive scan of the thread totals (warp 0 scans the warps)
      const unsigned long long incl = warp_incl_scan_u64(run);
      if (lane == 31) cs.wt[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        const unsigned long long t = cs.wt[lane];
        cs.wt[lane] = warp_incl_scan_u64(t) - t;
      }
      __syncthreads();
      const unsigned long long off = Ms + cs.wt[warp] + incl - run;
      // first stop and first hit of this segment
      int st = INT_MAX, fd = INT_MAX;
#pragma unroll
      for (int k = 0; k < kChainPer; k++) {
        const int j = j0 + k;
        if (j < cur || j >= wend || st != INT_MAX) continue;
        const unsigned long long m = off + pre[k];
        if (tie[k] || m >= 0x1000000ull) st = j;
        else if (MODE != kChainSum && fd == INT_MAX && chain_cond<MODE>(frecon(Es, m), target)) fd = j;
      }
      int S, Fd;
      block_min2(st, fd, cs, S, Fd);
      int next;
      if (Fd < S) {
        // a cumulative inside the segment meets the target
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == Fd) cs.sum = frecon(Es, off + pre[k]);
        found = Fd;
        next = wend;
      } else if (S == INT_MAX) {
        // no stop: the segment runs to the window's end
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == wend - 1) cs.sum = frecon(Es, off + pre[k]);
        next = wend;
      } else {
        // the stopping addend, by a real add from the exact cumulative before it
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == S) cs.sum = __fadd_rn(frecon(Es, off + pre[k] - nu[k]), v[k]);
        next = S + 1;
      }
      __syncthreads();
      s = cs.sum;
      __syncthreads();
      if (found < 0 && S != INT_MAX && Fd >= S && MODE != kChainSum && chain_cond<MODE>(s, target)) found = S;
      cur = next;
    }
  }
  if (hit) *hit = found;
  return s;
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

// Test hook: block_chain over n values in global memory (mode 0 sum, 1 first
// cumulative > target, 2 first cumulative >= target); out[0] = result,
// out[1] = hit index as float bits.
__global__ void __launch_bounds__(kSampThreads) chain_probe_kernel(const float* __restrict__ v, int n, int mode,
                                                                   float target, float* out) {
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  auto f = [&](int j) { return v[j]; };
  int hit = -1;
  float r;
  if (mode == 0) r = block_chain<kChainSum>(f, n, target, stage, sh, &hit);
  else if (mode == 1) r = block_chain<kChainFindLt>(f, n, target, stage, sh, &hit);
  else r = block_chain<kChainFindGe>(f, n, target, stage, sh, &hit);
  if (threadIdx.x == 0) {
    out[0] = r;
    out[1] = __int_as_float(hit);
  }
}

}  // namespace lz98
