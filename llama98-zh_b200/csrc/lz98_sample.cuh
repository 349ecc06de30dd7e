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
constexpr int kSortChunk = 8192;       // floats of dynamic shared memory (radix histograms)
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
// depend on s, except at an exact tie (v / u ending in .5), where the even
// rule adds floor(v / u) or one more by the parity of the running count.
// So inside a segment the running sum is s/u plus an integer prefix of
// per-addend counts, each a function of that parity (a pair: count when
// even, count when odd); pairs compose associatively, so the prefix is a
// parallel scan.  A segment ends at the first addend whose rounded prefix
// reaches the next binade (2^24 ulps); that addend is added with a real
// fadd and a new segment starts from the exact result.  Every cumulative
// equals the sequential one bit for bit (zeros keep s at 0; the first
// non-zero addend after them is taken exactly).
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

// Prefix sums of ulp counts saturate at 2^25: everything at or above 2^24
// ends the segment anyway, and saturating addition of non-negative
// numbers is associative, so the scans stay exact where they are used.
constexpr uint32_t kUlpSat = 1u << 25;
LZ_HD uint32_t sadd(uint32_t a, uint32_t b) { return min(a + b, kUlpSat); }

// ulps of v = Mj * 2^(Ej - 150) on the grid of exponent Es, without
// branches (the rounding of every addend of a window runs in one pass):
// shift right by r = Es - Ej (clamped to 31, zero when the addend's
// exponent is at or above the grid's), round half up, flag exact halves
// (tie); addends one binade above the grid double, two or more saturate.
LZ_HD uint32_t fulps_bf(int Ej, uint32_t Mj, int Es, bool& tie) {
  const int sh = Ej - Es;
  const uint32_t r = (uint32_t)min(max(-sh, 0), 31);
  const uint32_t rem = Mj & ((1u << r) - 1u);
  const uint32_t half = r ? 1u << (r - 1u) : 0u;
  tie = r != 0u && rem == half;
  const uint32_t down = (Mj >> r) + (rem > half ? 1u : 0u);
  const uint32_t up = sh >= 2 ? kUlpSat : min(Mj << 1, kUlpSat);
  return sh >= 1 ? up : down;
}

// The find condition on the grid of exponent Es: a cumulative m * u meets
// the target iff m > floor(target / u) (kChainFindLt) or m >= ceil(target /
// u) (kChainFindGe); returns that integer bound (target >= 0 here; a
// negative target is met by every cumulative).
template <int MODE>
LZ_HD int chain_bound(float target, int Es) {
  if (!(target >= 0.0f)) return MODE == kChainFindLt ? -1 : 0;
  int Et;
  uint32_t Mt;
  fdecomp(target, Et, Mt);
  const int sh = Et - Es;
  uint32_t fl, rem = 0;
  if (Mt == 0u) fl = 0u;
  else if (sh >= 0) fl = sh >= 2 ? kUlpSat : min(Mt << sh, kUlpSat);
  else if (-sh >= 25) { fl = 0u; rem = 1u; }
  else { fl = Mt >> -sh; rem = Mt & ((1u << -sh) - 1u); }
  if (MODE == kChainFindLt) return (int)fl;
  return (int)min(fl + (rem ? 1u : 0u), kUlpSat);
}

template <int MODE>
LZ_HD bool chain_cond(float c, float target) {
  return MODE == kChainFindLt ? (target < c) : (MODE == kChainFindGe ? (c >= target) : false);
}

constexpr int kChainHead = 1024;      // leading values summed serially
constexpr int kChainPer = 8;          // values per thread per window
constexpr int kChainWin = kChainPer * kSampThreads;
constexpr uint32_t kChainAll = (1u << kChainPer) - 1u;   // all of a thread's addends

// Composition of per-addend ulp counts that depend on the parity of the
// running count (a: count even before, b: odd): `x then y`.  Saturating,
// hence associative where it is used (below 2^24 ulps).
struct U2 {
  uint32_t a, b;
};
LZ_HD U2 u2_then(U2 x, U2 y) {
  return U2{sadd(x.a, (x.a & 1u) ? y.b : y.a), sadd(x.b, ((x.b + 1u) & 1u) ? y.b : y.a)};
}

LZ_HD U2 warp_incl_scan_u2(U2 v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const U2 w = {__shfl_up_sync(0xffffffffu, v.a, o), __shfl_up_sync(0xffffffffu, v.b, o)};
    if (lane >= o) v = u2_then(w, v);
  }
  return v;
}

struct ChainShared {
  U2 wt2[kSampWarps];                 // warp compositions, then exclusive prefixes
  uint32_t wt[kSampWarps];            // warp totals
  int wtie[kSampWarps];               // warp has a tie
  int wstop[kSampWarps], wfind[kSampWarps];
  int S, F;
  float sum;
  float sum2[2];                      // running sum after a round, by round parity
  int hit;
};

LZ_HD uint32_t warp_incl_scan_sat(uint32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t w = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = sadd(v, w);
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
// the total is returned.  The running sum starts at `init` (0 by default).  Every thread of the block calls it; `stage` holds
// kChainHead floats.
template <int MODE, class F>
__device__ float block_chain(F val, int n, float target, float* stage, SampShared& sh, int* hit, float init = 0.0f) {
  __shared__ ChainShared cs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // serial head: crossings are dense while the sum is small
  const int nh = min(n, kChainHead);
  for (int t = tid; t < nh; t += kSampThreads) stage[t] = val(t);
  __syncthreads();
  if (tid == 0) {
    float acc = init;
    int h = -1;
    int t = 0;
    // four addends per 16-byte load, the loads ahead of the adds; the find
    // modes test each cumulative in index order
#pragma unroll 4
    for (; t + 4 <= nh; t += 4) {
      const float4 q = *reinterpret_cast<const float4*>(stage + t);
      const float a0 = __fadd_rn(acc, q.x);
      const float a1 = __fadd_rn(a0, q.y);
      const float a2 = __fadd_rn(a1, q.z);
      const float a3 = __fadd_rn(a2, q.w);
      if (MODE != kChainSum) {
        const int c = chain_cond<MODE>(a0, target)   ? 0
                      : chain_cond<MODE>(a1, target) ? 1
                      : chain_cond<MODE>(a2, target) ? 2
                      : chain_cond<MODE>(a3, target) ? 3
                                                     : -1;
        if (c >= 0) {
          h = t + c;
          acc = c == 0 ? a0 : (c == 1 ? a1 : (c == 2 ? a2 : a3));
          break;
        }
      }
      acc = a3;
    }
    if (h < 0)
      for (; t < nh; t++) {
        acc = __fadd_rn(acc, stage[t]);
        if (MODE != kChainSum && chain_cond<MODE>(acc, target)) { h = t; break; }
      }
    cs.sum = acc;
    cs.hit = h;
  }
  __syncthreads();
  float s = cs.sum;
  int found = cs.hit;
  int par = 0;   // slot of cs.sum2 the next round writes
  for (int w0 = nh; w0 < n && found < 0; w0 += kChainWin) {
    const int j0 = w0 + tid * kChainPer;
    const int wend = min(n, w0 + kChainWin);
    float v[kChainPer];
    int ve[kChainPer];
    uint32_t vm[kChainPer];
    uint32_t inwin = 0u;               // this thread's addends inside the window
    int emax = 1;                      // their largest exponent
#pragma unroll
    for (int k = 0; k < kChainPer; k++) {
      v[k] = j0 + k < wend ? val(j0 + k) : 0.0f;
      fdecomp(v[k], ve[k], vm[k]);
      inwin |= j0 + k < wend ? 1u << k : 0u;
      emax = max(emax, ve[k]);
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
      // per addend its ulp count and whether it ties; a tie adds floor or
      // one more by the parity of the running count
      const int dc = cur - j0;         // this thread's addends before cur are closed
      const uint32_t livemask = dc <= 0 ? inwin : (dc >= kChainPer ? 0u : inwin & (kChainAll << dc));
      uint32_t qv[kChainPer];
      uint32_t tiemask = 0u;
      if (emax <= Es) {
        // every addend at or below the running sum's binade (the usual
        // case): round half up by the added half, less one at an exact
        // half, whose floor count the parity rule then settles
#pragma unroll
        for (int k = 0; k < kChainPer; k++) {
          const uint32_t r = (uint32_t)min(Es - ve[k], 31);
          const uint32_t p2 = 1u << r, half = p2 >> 1;
          const bool t = half != 0u && (vm[k] & (p2 - 1u)) == half;
          qv[k] = ((vm[k] + half) >> r) - (t ? 1u : 0u);
          tiemask |= t ? 1u << k : 0u;
        }
      } else {
#pragma unroll
        for (int k = 0; k < kChainPer; k++) {
          bool t;
          qv[k] = fulps_bf(ve[k], vm[k], Es, t);
          tiemask |= t ? 1u << k : 0u;
        }
      }
      tiemask &= livemask;
#pragma unroll
      for (int k = 0; k < kChainPer; k++) qv[k] = (livemask >> k) & 1u ? qv[k] : 0u;
      // plain saturating prefix sums first; the block learns at the same
      // barrier whether any addend of the window ties
      // (a thread's counts are each <= 2^25: eight of them stay below 2^28
      // without saturating; the warp and block sums saturate)
      uint32_t mk[kChainPer];
      uint32_t off;
      uint32_t run = 0u;
#pragma unroll
      for (int k = 0; k < kChainPer; k++) {
        run += qv[k];
        mk[k] = run;
      }
      const uint32_t incl = warp_incl_scan_sat(run);
      const bool wtie = __any_sync(0xffffffffu, tiemask != 0u);
      if (lane == 31) {
        cs.wt[warp] = incl;
        cs.wtie[warp] = wtie;
      }
      __syncthreads();
      if (!__any_sync(0xffffffffu, cs.wtie[lane] != 0)) {
        // every warp scans the 32 warp totals itself
        const uint32_t xw = warp_incl_scan_sat(cs.wt[lane]);
        const uint32_t wex = warp ? __shfl_sync(0xffffffffu, xw, warp - 1) : 0u;
        const uint32_t lb = __shfl_up_sync(0xffffffffu, incl, 1);
        off = sadd(sadd(Ms, wex), lane ? lb : 0u);
#pragma unroll
        for (int k = 0; k < kChainPer; k++) mk[k] += off;   // < 2^25 + 2^28: no wrap
      } else {
        // a parity function per addend (count if the running count is
        // even, count if odd), composed associatively
        U2 pre[kChainPer];
        U2 r2 = {0u, 0u};
#pragma unroll
        for (int k = 0; k < kChainPer; k++) {
          const uint32_t q = qv[k];
          const U2 d = ((tiemask >> k) & 1u) ? U2{q + (q & 1u), q + ((q + 1u) & 1u)} : U2{q, q};
          r2 = u2_then(r2, d);
          pre[k] = r2;
        }
        const U2 in2 = warp_incl_scan_u2(r2);
        if (lane == 31) cs.wt2[warp] = in2;
        __syncthreads();
        if (warp == 0) {
          const U2 x = warp_incl_scan_u2(cs.wt2[lane]);
          const U2 ex = {__shfl_up_sync(0xffffffffu, x.a, 1), __shfl_up_sync(0xffffffffu, x.b, 1)};
          cs.wt2[lane] = lane ? ex : U2{0u, 0u};
        }
        __syncthreads();
        // composition of everything before this thread, applied to Ms
        const U2 lb = {__shfl_up_sync(0xffffffffu, in2.a, 1), __shfl_up_sync(0xffffffffu, in2.b, 1)};
        const U2 before = u2_then(cs.wt2[warp], lane ? lb : U2{0u, 0u});
        off = sadd(Ms, (Ms & 1u) ? before.b : before.a);
        const uint32_t p1 = off & 1u;        // parity entering this thread's addends
#pragma unroll
        for (int k = 0; k < kChainPer; k++) mk[k] = sadd(off, p1 ? pre[k].b : pre[k].a);
      }
      const int bound = MODE == kChainSum ? 0 : chain_bound<MODE>(target, Es);
      uint32_t stopmask = 0u, hitmask = 0u;
#pragma unroll
      for (int k = 0; k < kChainPer; k++) {
        const uint32_t m = mk[k];
        stopmask |= m >= 0x1000000u ? 1u << k : 0u;
        if (MODE == kChainFindLt) hitmask |= (int)m > bound ? 1u << k : 0u;
        if (MODE == kChainFindGe) hitmask |= (int)m >= bound ? 1u << k : 0u;
      }
      stopmask &= livemask;
      hitmask &= livemask;
      const int st = stopmask ? j0 + __ffs(stopmask) - 1 : INT_MAX;
      int fd = hitmask ? j0 + __ffs(hitmask) - 1 : INT_MAX;
      if (fd >= st) fd = INT_MAX;
      // block minima: every warp reduces the 32 warp minima itself
      {
        const int ws = __reduce_min_sync(0xffffffffu, st), wf = __reduce_min_sync(0xffffffffu, fd);
        if (lane == 0) {
          cs.wstop[warp] = ws;
          cs.wfind[warp] = wf;
        }
      }
      __syncthreads();
      const int S = __reduce_min_sync(0xffffffffu, cs.wstop[lane]);
      const int Fd = __reduce_min_sync(0xffffffffu, cs.wfind[lane]);
      int next;
      float* nsum = &cs.sum2[par];
      if (Fd < S) {
        // a cumulative inside the segment meets the target
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == Fd) *nsum = frecon(Es, mk[k]);
        found = Fd;
        next = wend;
      } else if (S == INT_MAX) {
        // no stop: the segment runs to the window's end
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == wend - 1) *nsum = frecon(Es, mk[k]);
        next = wend;
      } else {
        // the addend that leaves the binade, by a real add from the exact
        // cumulative before it
#pragma unroll
        for (int k = 0; k < kChainPer; k++)
          if (j0 + k == S) *nsum = __fadd_rn(frecon(Es, k ? mk[k - 1] : off), v[k]);
        next = S + 1;
      }
      __syncthreads();
      s = *nsum;
      par ^= 1;   // the other slot next round: no barrier needed after the read
      if (found < 0 && S != INT_MAX && MODE != kChainSum && chain_cond<MODE>(s, target)) found = S;
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
  // the sum chain evaluates every exp exactly once; each is kept in out
  // and scaled there once the sum is known
  auto ev = [&](int j) {
    const float e = exp_body(__fsub_rn(__fmul_rn(__ldcg(lg + j), inv_t), mx));
    out[j] = e;
    return e;
  };
  const float sum = block_chain<kChainSum>(ev, n, 0.0f, stage, sh, nullptr);
  const float invs = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
  for (int j = threadIdx.x; j < n; j += kSampThreads) out[j] = __fmul_rn(out[j], invs);
  __syncthreads();
}

// Exclusive scan over the block's threads in index order (every thread
// calls; `id` is the value before thread 0), with the block total.
template <class Op>
__device__ uint32_t block_excl_scan_u32(uint32_t v, uint32_t id, Op op, uint32_t* total) {
  __shared__ uint32_t wsh[kSampWarps];
  static_assert(kSampWarps == 32, "one warp scans the warp totals");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t w = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x = op(w, x);
  }
  __syncthreads();
  if (lane == 31) wsh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t t = wsh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t w = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t = op(w, t);
    }
    wsh[lane] = t;
  }
  __syncthreads();
  const uint32_t wex = warp ? op(id, wsh[warp - 1]) : id;
  const uint32_t lex = __shfl_up_sync(0xffffffffu, x, 1);
  if (total) *total = op(id, wsh[kSampWarps - 1]);
  __syncthreads();
  return lane ? op(wex, lex) : wex;
}

// lz_argmax_p1 (src/sampler.c:279-295): the first index of the maximum (by
// `>`) and 1 / l, l the online softmax normaliser: l starts at 1 for
// element 0; a new running maximum v rescales it, l = l * exp(best - v) + 1;
// every other element adds exp(v - best) in index order.  The positions of
// the running maxima (records) are found by a block scan and written to
// recs (n ints); the sums between records run as exact sequential chains
// from the current l.  Every thread calls; all get the result.
__device__ int block_argmax_p1(const float* __restrict__ lg, int n, float* p1, int* recs, float* stage, SampShared& sh) {
  __shared__ int nrec_s;
  const int tid = threadIdx.x;
  const int per = (n + kSampThreads - 1) / kSampThreads;
  const int a = min(n, tid * per), b = min(n, a + per);
  uint32_t mk = 0u;
  for (int i = a; i < b; i++) {
    const uint32_t k = fkey(lg[i]);
    mk = k > mk ? k : mk;
  }
  auto umax = [](uint32_t x, uint32_t y) { return x > y ? x : y; };
  const uint32_t before = block_excl_scan_u32(mk, 0u, umax, nullptr);
  // records of this thread's range, counted then written in order
  auto walk = [&](int* out) {
    int c = 0;
    float run;
    int i0 = a;
    if (a == 0) {
      run = lg[0];
      i0 = 1;
    } else {
      run = key_float(before);
    }
    for (int i = i0; i < b; i++) {
      const float v = lg[i];
      if (v > run) {
        if (out) out[c] = i;
        c++;
        run = v;
      }
    }
    return c;
  };
  const int cnt = a < b ? walk(nullptr) : 0;
  uint32_t tot;
  const uint32_t off = block_excl_scan_u32((uint32_t)cnt, 0u, [](uint32_t x, uint32_t y) { return x + y; }, &tot);
  if (a < b) walk(recs + off);
  if (tid == 0) nrec_s = (int)tot;
  __syncthreads();
  const int nrec = nrec_s;
  float l = 1.0f, best = lg[0];
  int prev = 0;
  for (int j = 0; j <= nrec; j++) {
    const int r = j < nrec ? recs[j] : n;
    const int len = r - prev - 1;
    if (len > 0) {
      const float bb = best;
      const int p0 = prev + 1;
      auto ev = [&](int t) { return exp_body(__fsub_rn(__ldcg(lg + p0 + t), bb)); };
      l = block_chain<kChainSum>(ev, len, 0.0f, stage, sh, nullptr, l);
    }
    if (j < nrec) {
      const float v = lg[r];
      l = __fadd_rn(__fmul_rn(l, exp_body(__fsub_rn(best, v))), 1.0f);
      best = v;
      prev = r;
    }
  }
  *p1 = l > 0.0f ? __fdiv_rn(1.0f, l) : 1.0f;
  __syncthreads();
  return prev;
}

// First index of the maximum by order key (src/sampler.c:224-240).
__device__ int block_argmax(const float* v, int n, SampShared& sh) {
  unsigned long long best = 0ull;
  for (int j = threadIdx.x; j < n; j += kSampThreads) {
    const unsigned long long k = ((unsigned long long)fkey(__ldcg(v + j)) << 32) | (uint32_t)~(uint32_t)j;
    best = k > best ? k : best;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  best = warp_max_u64(best);
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

// Descending sort of n non-negative floats by one block: a stable LSD radix
// sort on the complemented bit patterns (4 passes of 8 bits; for floats
// >= 0 the bit pattern orders like the value).  a holds the keys ~bits(v)
// on entry (0xFFFFFFFF for entries that must sort last) and the sorted
// values on exit; tmp is n words of scratch; hist is 32 x 256 words of
// shared memory.  Each warp owns a contiguous chunk and walks it in order,
// ranking equal digits within the warp by ballots, so every pass is stable.
// Lanes of the warp holding the same 8-bit digit (among lanes with ok set):
// the intersection over the digit's bits of the ballot of that bit or of
// its complement.
LZ_HD unsigned digit_peers(uint32_t d, bool ok) {
  unsigned m = __ballot_sync(0xffffffffu, ok);
#pragma unroll
  for (int b = 0; b < 8; b++) {
    const unsigned v = __ballot_sync(0xffffffffu, (d >> b) & 1u);
    m &= ((d >> b) & 1u) ? v : ~v;
  }
  return m;
}

__device__ void block_radix_sort_desc(uint32_t* a, uint32_t* tmp, int n, uint32_t* hist) {
  constexpr int U = 16;                // keys per lane loaded ahead of the in-order walk
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = ((n + kSampWarps - 1) / kSampWarps + 32 * U - 1) / (32 * U) * (32 * U);
  const int c0 = min(n, warp * chunk), c1 = min(n, c0 + chunk);
  const unsigned lt = (1u << lane) - 1u;
  uint32_t* src = a;
  uint32_t* dst = tmp;
  for (int pass = 0; pass < 4; pass++) {
    const int shift = pass * 8;
    for (int i = tid; i < kSampWarps * 256; i += kSampThreads) hist[i] = 0u;
    __syncthreads();
    uint32_t* h = hist + warp * 256;
    // the warp's digit counts (its own histogram: the order of the adds
    // does not matter)
    for (int i0 = c0; i0 < c1; i0 += 32 * U) {
      uint32_t kk[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int i = i0 + u * 32 + lane;
        kk[u] = i < c1 ? __ldcg(src + i) : 0u;
      }
#pragma unroll
      for (int u = 0; u < U; u++)
        if (i0 + u * 32 + lane < c1) atomicAdd(&h[(kk[u] >> shift) & 255u], 1u);
    }
    __syncthreads();
    // exclusive offsets per (warp, digit): digit bases in digit order, then
    // the warps in chunk order
    if (tid < 256) {
      uint32_t t = 0;
      for (int w = 0; w < kSampWarps; w++) t += hist[w * 256 + tid];
      uint32_t x = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      __shared__ uint32_t wsum[8];
      if (lane == 31) wsum[warp] = x;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      uint32_t base = x - t;
      for (int w = 0; w < warp; w++) base += wsum[w];
      for (int w = 0; w < kSampWarps; w++) {
        const uint32_t c = hist[w * 256 + tid];
        hist[w * 256 + tid] = base;
        base += c;
      }
    }
    __syncthreads();
    for (int i0 = c0; i0 < c1; i0 += 32 * U) {
      uint32_t kk[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int i = i0 + u * 32 + lane;
        kk[u] = i < c1 ? __ldcg(src + i) : 0u;
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const bool ok = i0 + u * 32 + lane < c1;
        const uint32_t d = (kk[u] >> shift) & 255u;
        const unsigned peers = digit_peers(d, ok);
        if (ok) dst[h[d] + __popc(peers & lt)] = pass == 3 ? ~kk[u] : kk[u];
        __syncwarp();
        if (ok && (peers & lt) == 0u) h[d] += __popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
    uint32_t* t2 = src;
    src = dst;
    dst = t2;
  }
  // four passes: the result is back in a (as value bits)
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
// 2 * npow2 floats (sorted candidates first); returns the nucleus.
__device__ Nucleus block_nucleus(const float* p, int n, float topp, float* sorted, int npow2, float* stage,
                                 SampShared& sh) {
  const float cut = n > 1 ? __fdiv_rn(__fsub_rn(1.0f, topp), (float)(n - 1)) : 0.0f;
  uint32_t* keys = reinterpret_cast<uint32_t*>(sorted);
  int cnt = 0;
  for (int j = threadIdx.x; j < n; j += kSampThreads) {
    const float v = p[j];
    const bool c = v >= cut;
    keys[j] = c ? ~__float_as_uint(v) : 0xFFFFFFFFu;
    cnt += c;
  }
  Nucleus nu;
  nu.n0 = block_sum_i(cnt, sh);
  nu.last = -1;
  nu.mass = 0.0f;
  if (nu.n0 <= 0) return nu;
  block_radix_sort_desc(keys, keys + npow2, n, reinterpret_cast<uint32_t*>(stage));
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
// 2 * npow2 floats of scratch.
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
  // every element equal to v_last kept (the usual case): no ordered count
  int eq_all = 0;
  for (int j = threadIdx.x; j < n; j += kSampThreads) eq_all += p[j] == vl;
  if (block_sum_i(eq_all, sh) <= need) {
    for (int j = threadIdx.x; j < n; j += kSampThreads) {
      const float v = p[j];
      p[j] = v >= vl ? __fdiv_rn(v, nu.mass) : 0.0f;
    }
    __syncthreads();
    return;
  }
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
// scratch rows (n and 2 * npow2 floats).  Thread 0 owns *rng.
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

// One greedy draft step's arg-max with its lz_argmax_p1 probability (the
// confidence p_min is compared with, src/generate.c:756-762): sequence 0's
// logits row; the token goes to sr[0].draft[i], the probability to conf[0].
__global__ void __launch_bounds__(kSampThreads) argmax_p1_kernel(const float* __restrict__ logits, int V,
                                                                SeqRound* sr, int i, int k, int* recs,
                                                                float* conf) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  float p1;
  const int idx = block_argmax_p1(logits, V, &p1, recs, stage, sh);
  if (threadIdx.x == 0) {
    sr[0].draft[i] = idx;
    sr[0].k = k;
    conf[0] = p1;
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
                    sortbuf + (size_t)row * 2 * npow2, npow2, stage, sh);
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

// Test hook: lz_argmax_p1 of one row (out[0] = probability, out[1] = index bits).
__global__ void __launch_bounds__(kSampThreads) argmax_p1_probe_kernel(const float* __restrict__ v, int n, int* recs,
                                                                      float* out) {
  extern __shared__ __align__(16) float stage[];
  __shared__ SampShared sh;
  float p1;
  const int idx = block_argmax_p1(v, n, &p1, recs, stage, sh);
  if (threadIdx.x == 0) {
    out[0] = p1;
    out[1] = __int_as_float(idx);
  }
}

}  // namespace lz98
