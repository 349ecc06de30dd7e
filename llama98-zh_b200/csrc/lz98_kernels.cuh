// CUDA kernels of the MTP speculative-decoding step (sm_100a).
//
// Layout in HBM (all row-major):
//   activations  x  f32 [R][d]           one row per (sequence, position)
//   quantised    xq i8  [R][K], xs f32 [R][K/32]   (per-32 absmax/127)
//   Q8_0 weight  W  i8  [N][K], ws f32 [N][K/gs]    (gs = 32 or K)
//   KDA state    hi/lo i8 [seq][ring][layer][head][64][64],
//                scale f32 [seq][ring][layer][head][64][2]
//   conv state   f32 [seq][ring][layer][3*H*64][3]
//   MTP KV cache kq/vq i8 [seq][pos][kv_dim], ks/vs f32 [seq][pos][kv_dim/32]
//
// Every float reduction keeps the reference's order: where the reference
// sums sequentially the kernel sums sequentially (one lane per chain, the
// chains of different rows/columns in parallel, operands staged in shared
// memory so the chain runs at add latency); integer sums (int8 dot
// products per 32-element sub-block) are order-free and run as __dp4a.
#pragma once
#include <cuda.h>   // CUtensorMap (the type only; maps are encoded through the runtime's driver entry point)
#include "lz98_dev.cuh"

namespace lz98 {

constexpr int kGemvWarps = 4;
constexpr int kGemvProWarps = 16;   // warps of a GEMV block that runs the input-norm prologue
constexpr int kGemvRB = 8;        // token rows per reduction pass
constexpr int kRowLoadU = 4;      // loads a thread of a row kernel issues before its stores

// ------------------------------------------------------- serial chains

// Sequential sum of squares over a 16-byte aligned array, n % 4 == 0
// (src/ops_norm.c:718): the adds stay in index order; the loads run ahead
// in float4 groups.  (Forming 16 squares ahead of the chain measured
// faster alone but slower inside the 128-register prologue GEMV.)
LZ_HD float seq_sumsq(const float* v, int n) {
  float ss = 0.0f;
  const float4* p = reinterpret_cast<const float4*>(v);
#pragma unroll 8
  for (int i = 0; i < n / 4; i++) {
    const float4 q = p[i];
    ss = __fadd_rn(ss, __fmul_rn(q.x, q.x));
    ss = __fadd_rn(ss, __fmul_rn(q.y, q.y));
    ss = __fadd_rn(ss, __fmul_rn(q.z, q.z));
    ss = __fadd_rn(ss, __fmul_rn(q.w, q.w));
  }
  return ss;
}

// The same sequential sum of squares over a row of K floats (K % 512 == 0)
// by a group of 128 threads, in about half the chain's time.  The row
// splits into four segments.  The group squares the row into `sq` (one
// segment per warp, each segment padded by 16 bytes so the segments sit on
// different banks) and sums each segment's squares as a float tree.  Two
// warps of the group then run the chains, two per lane on each loaded
// square: lane 0 the first segment's chain from zero, the other lanes the
// later segments' chains from candidate starts - the consecutive floats
// around the segment's prefix of tree sums (32, 32 and 62 of them).  The
// sequential prefix departs from that estimate by a few units in the last
// place (under half an ulp per add, a random walk), so one candidate
// almost always starts exactly from it.  Lane 0 walks the segments: the
// candidate whose start equals the prefix reached so far is found by
// index, and a segment with no such candidate is chained by lane 0 itself.
// The result is the sequential sum bit for bit (src/ops_norm.c:718).
// (Shared-memory bandwidth bounds the chains: each lane reads its whole
// segment, so two chains per lane halve the bytes of one.)
//   x: the row in shared memory (16-byte aligned); sq: shared scratch of
//   K + 16 floats; u: the thread's index in the group; cw: the first of
//   the two chain warps (0 or 2); r: the group (0-3), which names its
//   barriers.  Returns the sum in lane 0 of warp cw (0 elsewhere).
constexpr int kSplitGroup = 128;
// 16-byte aligned: the chain lanes store their two ends as one float2
struct __align__(16) SplitSumShared {
  float part[4];
  float end[128];
};

// named barriers with immediate ids: the group's 128 threads (ids 1-4),
// then its two chain warps (ids 5-8)
LZ_HD void group_bar(int r) {
  switch (r) {
    case 0: asm volatile("bar.sync 1, 128;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 2, 128;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 3, 128;" ::: "memory"); break;
    default: asm volatile("bar.sync 4, 128;" ::: "memory"); break;
  }
}
LZ_HD void chain_bar(int r) {
  switch (r) {
    case 0: asm volatile("bar.sync 5, 64;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 6, 64;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 7, 64;" ::: "memory"); break;
    default: asm volatile("bar.sync 8, 64;" ::: "memory"); break;
  }
}

LZ_HD float seq_sumsq_split(const float* x, float* sq, int K, int u, int cw, int r, SplitSumShared& sh) {
  const int L = K / 4, LP = L + 4, per = K / kSplitGroup, su = u >> 5;
  float acc = 0.0f;
  for (int i = u * per; i < (u + 1) * per; i += 4) {
    const float4 q = *reinterpret_cast<const float4*>(x + i);
    const float4 p = make_float4(__fmul_rn(q.x, q.x), __fmul_rn(q.y, q.y), __fmul_rn(q.z, q.z), __fmul_rn(q.w, q.w));
    *reinterpret_cast<float4*>(sq + su * LP + (i - su * L)) = p;
    acc = __fadd_rn(acc, __fadd_rn(__fadd_rn(p.x, p.y), __fadd_rn(p.z, p.w)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  if ((u & 31) == 0) sh.part[su] = acc;
  group_bar(r);
  const int t = u - 32 * cw;            // chain lane, 0-63
  if (t < 0 || t >= 64) return 0.0f;
  const float g1 = sh.part[0], g2 = __fadd_rn(g1, sh.part[1]), g3 = __fadd_rn(g2, sh.part[2]);
  int seg = 0, o = 0;
  float g = 0.0f;
  if (t >= 33) seg = 3, g = g3, o = 2 * (t - 33) - 31;
  else if (t >= 17) seg = 2, g = g2, o = 2 * (t - 17) - 16;
  else if (t >= 1) seg = 1, g = g1, o = 2 * (t - 1) - 16;
  float c0 = 0.0f, c1 = 0.0f;
  if (t > 0) {
    c0 = __int_as_float(__float_as_int(g) + o);
    c1 = __int_as_float(__float_as_int(g) + o + 1);
  }
  const float4* p = reinterpret_cast<const float4*>(sq + seg * LP);
#pragma unroll 4
  for (int i = 0; i < L / 4; i++) {
    const float4 q = p[i];
    c0 = __fadd_rn(c0, q.x);
    c1 = __fadd_rn(c1, q.x);
    c0 = __fadd_rn(c0, q.y);
    c1 = __fadd_rn(c1, q.y);
    c0 = __fadd_rn(c0, q.z);
    c1 = __fadd_rn(c1, q.z);
    c0 = __fadd_rn(c0, q.w);
    c1 = __fadd_rn(c1, q.w);
  }
  *reinterpret_cast<float2*>(&sh.end[2 * t]) = make_float2(c0, c1);
  chain_bar(r);
  if (t != 0) return 0.0f;
  float v = c0;
  const float gs[3] = {g1, g2, g3};
  const int first[3] = {2, 34, 66}, ctr[3] = {16, 16, 31}, nc[3] = {32, 32, 62};
#pragma unroll
  for (int s = 0; s < 3; s++) {
    const int d = __float_as_int(v) - __float_as_int(gs[s]) + ctr[s];
    if ((unsigned)d < (unsigned)nc[s]) {
      v = sh.end[first[s] + d];
    } else {   // no candidate started from the prefix: chain the segment here
      const float* ps = sq + (s + 1) * LP;
      for (int i = 0; i < L; i++) v = __fadd_rn(v, ps[i]);
    }
  }
  return v;
}

// Test probe of seq_sumsq_split: one 128-thread group per row (up to 4
// rows of n floats), the rows and their squares in dynamic shared memory.
__global__ void sumsq_split_probe_kernel(const float* __restrict__ rows, int nrows, int n, float* out) {
  extern __shared__ __align__(16) float psm[];
  __shared__ SplitSumShared sh[4];
  float* x = psm;
  float* sq = psm + (size_t)nrows * n;
  for (int i = threadIdx.x; i < nrows * n; i += blockDim.x) x[i] = rows[i];
  __syncthreads();
  const int r = threadIdx.x / kSplitGroup, u = threadIdx.x - r * kSplitGroup, cw = 2 * (r & 1);
  const float v = seq_sumsq_split(x + (size_t)r * n, sq + (size_t)r * (n + 16), n, u, cw, r, sh[r]);
  if (u == 32 * cw) out[r] = v;
}

// Sequential sum (index order) of a 16-byte aligned array, any n.
LZ_HD float seq_sum(const float* v, int n) {
  float s = 0.0f;
  const float4* p = reinterpret_cast<const float4*>(v);
  int i = 0;
#pragma unroll 8
  for (; i < n / 4; i++) {
    const float4 q = p[i];
    s = __fadd_rn(s, q.x);
    s = __fadd_rn(s, q.y);
    s = __fadd_rn(s, q.z);
    s = __fadd_rn(s, q.w);
  }
  for (i *= 4; i < n; i++) s = __fadd_rn(s, v[i]);
  return s;
}

// ------------------------------------------------------------------ GEMV

// The float reduction of one output element from its per-32 products,
// src/ops_matmul.c:590-629 / src/ops_epi.c:983-1023:
//   rb = gs/32 > 1: p[s] = acc[s]*xs[s]; sum over groups of (sum of p in the
//                   group) * ws[g], both sequential;
//   rb == 1:        p[s] = acc[s]*(xs[s]*ws[s]); four interleaved
//                   accumulators combined (a0+a2)+(a1+a3), tail into a0.
// p is 16-byte aligned.
LZ_HD float q8_reduce(const float* p, const float* wsr, int rb, int ng) {
  if (rb > 1) {
    if (ng == 1) return __fadd_rn(0.0f, __fmul_rn(seq_sum(p, rb), wsr[0]));
    float sum = 0.0f;
    for (int g = 0; g < ng; g++) {
      float dot = 0.0f;
      for (int s = 0; s < rb; s++) dot = __fadd_rn(dot, p[g * rb + s]);
      sum = __fadd_rn(sum, __fmul_rn(dot, wsr[g]));
    }
    return sum;
  }
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  int g = 0;
  const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll 4
  for (; g + 3 < ng; g += 4) {
    const float4 q = p4[g >> 2];
    a0 = __fadd_rn(a0, q.x);
    a1 = __fadd_rn(a1, q.y);
    a2 = __fadd_rn(a2, q.z);
    a3 = __fadd_rn(a3, q.w);
  }
  for (; g < ng; g++) a0 = __fadd_rn(a0, p[g]);
  return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}

// q8_reduce over products stored with a stride (p[s * ld], the GEMV's
// transposed product buffer), the same float operations in the same order;
// s0 is ws[0], already loaded, for one group per row (rb > 1, ng == 1).
LZ_HD float q8_reduce_st(const float* p, int ld, const float* wsr, float s0, int rb, int ng) {
  if (rb > 1) {
    if (ng == 1) {
      float sum = 0.0f;
#pragma unroll 8
      for (int s = 0; s < rb; s++) sum = __fadd_rn(sum, p[s * ld]);
      return __fadd_rn(0.0f, __fmul_rn(sum, s0));
    }
    float sum = 0.0f;
    for (int g = 0; g < ng; g++) {
      float dot = 0.0f;
      for (int s = 0; s < rb; s++) dot = __fadd_rn(dot, p[(g * rb + s) * ld]);
      sum = __fadd_rn(sum, __fmul_rn(dot, wsr[g]));
    }
    return sum;
  }
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  int g = 0;
#pragma unroll 4
  for (; g + 3 < ng; g += 4) {
    a0 = __fadd_rn(a0, p[g * ld]);
    a1 = __fadd_rn(a1, p[(g + 1) * ld]);
    a2 = __fadd_rn(a2, p[(g + 2) * ld]);
    a3 = __fadd_rn(a3, p[(g + 3) * ld]);
  }
  for (; g < ng; g++) a0 = __fadd_rn(a0, p[g * ld]);
  return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}

// The exact int32 dot product of a 32-element sub-block: two independent
// __dp4a chains (its dependent latency is ~13 cycles here) joined by one
// add; integer sums are exact in any order.
LZ_HD int dot32(const int4 wa, const int4 wb, const int4 xa, const int4 xb) {
  int a0 = __dp4a(wa.x, xa.x, 0), a1 = __dp4a(wb.x, xb.x, 0);
  a0 = __dp4a(wa.y, xa.y, a0); a1 = __dp4a(wb.y, xb.y, a1);
  a0 = __dp4a(wa.z, xa.z, a0); a1 = __dp4a(wb.z, xb.z, a1);
  a0 = __dp4a(wa.w, xa.w, a0); a1 = __dp4a(wb.w, xb.w, a1);
  return a0 + a1;
}

struct SeqRound;
struct MtpRow;

// The fused greedy tail of an lm_head GEMV of at most 8 token rows (the
// logits-to-acceptance path of a greedy round): every block folds the
// arg-max of its outputs per token row into amax (the packed order key of
// argmax_kernel, one atomic per block and row; the slots are cleared by
// an earlier kernel of the round), and, when sr is set, the last block to
// finish runs the round's acceptance (spec_accept_greedy_kernel's work)
// for every sequence.
struct GemvFuse {
  unsigned long long* amax;   // nullptr: off
  int p1;                     // -0 compares equal to +0 (the draft steps)
  SeqRound* sr; int nseq, kmax;
  const float* vhid; int d; float* chain; int depth, seq_len;
  MtpRow* catch_rows; int* catch_tok; int* catch_hidx;
  int* counter;
};
LZ_HD void greedy_accept_all(const GemvFuse& f);

struct GemvArgs {
  const int8_t* W; const float* ws; int N, K, gs;
  const int8_t* xq; const float* xs; int R;      // quantised input rows
  float* y; int ldy; int mode;        // mode 0: y = v; mode 1: y = y + v
  // optional second product over the same output rows, added before the
  // store: v = v1 + v2 (up projection plus shared expert,
  // src/forward_moe.c:434-545)
  const int8_t* W2; const float* ws2; int K2, gs2;
  const int8_t* xq2; const float* xs2;
  // optional input-norm prologue (R <= kGemvRB): every block normalises the
  // R float rows of nx (length K) with RMSNorm (1+nw) and quantises them
  // per 32 into shared memory; block 0 also stores the normalised rows to
  // nout and clears the arg-max slots namax.
  const float* nx; const float* nw; float eps; float* nout; unsigned long long* namax;
  GemvFuse fz;               // fused arg-max / acceptance (input-norm path only)
};

// Four 32-element groups at once (one element of each per lane): the
// reference quantiser (src/ops_quant.c:2152-2282) with the four max
// reductions interleaved.
LZ_HD void warp_quant32_x4(const float* v, int8_t* q, float* sg) {
  uint32_t m[4];
#pragma unroll
  for (int k = 0; k < 4; k++) m[k] = abs_bits(v[k]);
#pragma unroll
  for (int k = 0; k < 4; k++) m[k] = __reduce_max_sync(0xffffffffu, m[k]);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    float inv;
    q8_scale_from_amax(m[k], &sg[k], &inv);
    q[k] = (int8_t)q8_clamp(q8_round(__fmul_rn(v[k], inv)));
  }
}

// One weight row held in registers: the lane's 32-byte sub-blocks and,
// for gs = 32, their scales.
template <int JM>
struct WRow {
  int4 a[JM], b[JM];
  float s[JM];
};

template <int JM>
LZ_HD void load_wrow(WRow<JM>& w, const int8_t* __restrict__ wr, const float* __restrict__ wsr, int K, int rb,
                     int lane) {
  const int nsb = K >> 5;
#pragma unroll
  for (int j = 0; j < JM; j++) {
    const int s = lane + 32 * j;
    if (s < nsb) {
      w.a[j] = __ldg(reinterpret_cast<const int4*>(wr + s * 32));
      w.b[j] = __ldg(reinterpret_cast<const int4*>(wr + s * 32 + 16));
      w.s[j] = rb == 1 ? __ldg(wsr + s) : 0.0f;
    }
  }
}

// Products of NR weight rows (the first nvalid of them) with every token
// row for this lane's sub-blocks: every activation load and every product
// comes before the first store to P, so the stores (which may alias the
// activations in shared memory) never stall the next loads.  P is
// transposed: P[s * ld + i * nr + rr] receives the product of sub-block s
// of weight row i with token row rr (ld odd, so both these stores and the
// reducing lanes' reads along s are free of bank conflicts).
template <int JM, bool SH, int RB, int NR>
LZ_HD void gemv_products_nr(const WRow<JM> (&w)[NR], int nvalid, int K, int rb, const int8_t* xq, const float* xs,
                            int nr, float* P, int ld, int lane) {
  const int nsb = K >> 5;
  float pr[RB][NR][JM];
#pragma unroll
  for (int rr = 0; rr < RB; rr++) {
    if (rr < nr) {
      const int8_t* xr = xq + (size_t)rr * K;
      const float* xsr = xs + (size_t)rr * nsb;
#pragma unroll
      for (int j = 0; j < JM; j++) {
        const int s = lane + 32 * j;
        if (s < nsb) {
          int4 xa, xb;
          float xsv;
          if (SH) {
            xa = *reinterpret_cast<const int4*>(xr + s * 32);
            xb = *reinterpret_cast<const int4*>(xr + s * 32 + 16);
            xsv = xsr[s];
          } else {
            xa = __ldg(reinterpret_cast<const int4*>(xr + s * 32));
            xb = __ldg(reinterpret_cast<const int4*>(xr + s * 32 + 16));
            xsv = __ldg(xsr + s);
          }
#pragma unroll
          for (int i = 0; i < NR; i++)
            if (i < nvalid) {
              const float a = (float)dot32(w[i].a[j], w[i].b[j], xa, xb);
              pr[rr][i][j] = rb > 1 ? __fmul_rn(a, xsv) : __fmul_rn(a, __fmul_rn(xsv, w[i].s[j]));
            }
        }
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < RB; rr++)
#pragma unroll
    for (int i = 0; i < NR; i++)
#pragma unroll
      for (int j = 0; j < JM; j++) {
        const int s = lane + 32 * j;
        if (rr < nr && i < nvalid && s < nsb) P[s * ld + i * nr + rr] = pr[rr][i][j];
      }
}

// Weight rows a warp takes per step on the multi-row path.
template <int JM>
__host__ __device__ constexpr int gemv_nr() { return 4 / JM; }

// Bytes of dynamic shared memory of one GEMV block: per-warp product
// buffers, transposed with an odd stride (multi-row path: RB x NR
// columns + 1; single-row path: 8 + 1 columns for each of the two
// weights) and, with the input-norm prologue, the rows, norm weights,
// quantised rows, scales and inverse norms.
inline size_t gemv_smem_bytes(int JM, int warps, int RB, bool single, bool prologue, int R, int K) {
  size_t b = single ? (size_t)warps * 2 * (kGemvRB + 1) * JM * 32 * 4
                    : (size_t)warps * (RB * (4 / JM) + 1) * JM * 32 * 4;
  if (prologue) b += (size_t)R * K * 4 + (size_t)K * 4 + (size_t)R * K + (size_t)R * (K / 32) * 4 + 64;
  return b;
}

// One output row per step, any number of token rows (8 at a time) and an
// optional second weight over the same outputs.
template <int JM, int WARPS, bool SH>
LZ_HD void gemv_rows(const GemvArgs& a, const int8_t* xq, const float* xs, WRow<JM>& wn1, WRow<JM>& wn2,
                     float* P, float* P2, int n, int lane, float s1_first, float s2_first) {
  constexpr int LD = kGemvRB + 1;
  const int n_first = n;
  const int rb = a.gs >> 5, ng = a.K / a.gs;
  const int rb2 = a.W2 ? a.gs2 >> 5 : 0, ng2 = a.W2 ? a.K2 / a.gs2 : 0;
  const int nstep = gridDim.x * WARPS;
  for (; n < a.N; n += nstep) {
    const WRow<JM> w1 = wn1, w2 = wn2;
    if (n + nstep < a.N) {                 // the next row's weights stay in flight
      load_wrow<JM>(wn1, a.W + (size_t)(n + nstep) * a.K, a.ws + (size_t)(n + nstep) * ng, a.K, rb, lane);
      if (a.W2) load_wrow<JM>(wn2, a.W2 + (size_t)(n + nstep) * a.K2, a.ws2 + (size_t)(n + nstep) * ng2, a.K2, rb2, lane);
    }
    const float* wsr = a.ws + (size_t)n * ng;
    const float* wsr2 = a.W2 ? a.ws2 + (size_t)n * ng2 : nullptr;
    // the output row's scales (one per row) for the reducing lanes (the
    // first row's loaded before the dependency wait)
    const float s1 = n == n_first ? s1_first : (rb > 1 && ng == 1) ? __ldg(wsr) : 0.0f;
    const float s2 = n == n_first ? s2_first : (a.W2 && rb2 > 1 && ng2 == 1) ? __ldg(wsr2) : 0.0f;
    for (int r0 = 0; r0 < a.R; r0 += kGemvRB) {
      const int nr = min(kGemvRB, a.R - r0);
      float prev = 0.0f;
      if (lane < nr && a.mode == 1) prev = a.y[(size_t)(r0 + lane) * a.ldy + n];
      const WRow<JM> w1a[1] = {w1};
      gemv_products_nr<JM, SH, kGemvRB, 1>(w1a, 1, a.K, rb, xq + (size_t)r0 * a.K, xs + (size_t)r0 * (a.K >> 5), nr,
                                          P, LD, lane);
      if (a.W2) {
        const WRow<JM> w2a[1] = {w2};
        gemv_products_nr<JM, false, kGemvRB, 1>(w2a, 1, a.K2, rb2, a.xq2 + (size_t)r0 * a.K2,
                                               a.xs2 + (size_t)r0 * (a.K2 >> 5), nr, P2, LD, lane);
      }
      __syncwarp();
      if (lane < nr) {
        float v = q8_reduce_st(P + lane, LD, wsr, s1, rb, ng);
        if (a.W2) v = __fadd_rn(v, q8_reduce_st(P2 + lane, LD, wsr2, s2, rb2, ng2));
        a.y[(size_t)(r0 + lane) * a.ldy + n] = a.mode == 1 ? __fadd_rn(prev, v) : v;
      }
      __syncwarp();
    }
  }
}

// Rows of one warp taken NR at a time (weights of the next NR rows in
// flight while these compute): the products of all NR rows x R token rows
// (R <= RB <= 8), then their NR * R reductions on as many lanes at once.
template <int JM, int WARPS, bool SH, int RB>
LZ_HD void gemv_rows_multi(const GemvArgs& a, const int8_t* xq, const float* xs, WRow<JM> (&wc)[gemv_nr<JM>()],
                           float* P, int n0, int lane, float s0_first, unsigned long long& kbest) {
  constexpr int NR = gemv_nr<JM>(), LD = RB * NR + 1;
  const int rb = a.gs >> 5, ng = a.K / a.gs, R = a.R;
  const int nstep = gridDim.x * WARPS;
  WRow<JM> wn[NR];
  for (int base = n0; base < a.N; base += NR * nstep) {
    const int nb = base + NR * nstep;
#pragma unroll
    for (int i = 0; i < NR; i++) {
      const int r = nb + i * nstep;
      if (r < a.N) load_wrow<JM>(wn[i], a.W + (size_t)r * a.K, a.ws + (size_t)r * ng, a.K, rb, lane);
    }
    // the reducing lane's output row scale (one per row) and accumulator
    // input, loaded before the products
    const int li = lane / R, lrr = lane - li * R, lr = base + li * nstep;
    const bool red = lane < NR * R && lr < a.N;
    float s0 = 0.0f, prev = 0.0f;
    if (red) {
      if (rb > 1 && ng == 1) s0 = base == n0 ? s0_first : __ldg(a.ws + lr);
      if (a.mode == 1) prev = a.y[(size_t)lrr * a.ldy + lr];
    }
    const int nvalid = base >= a.N ? 0 : min(NR, (a.N - 1 - base) / nstep + 1);
    gemv_products_nr<JM, SH, RB, NR>(wc, nvalid, a.K, rb, xq, xs, R, P, LD, lane);
    __syncwarp();
    if (red) {
      const float v = q8_reduce_st(P + lane, LD, a.ws + (size_t)lr * ng, s0, rb, ng);
      a.y[(size_t)lrr * a.ldy + lr] = a.mode == 1 ? __fadd_rn(prev, v) : v;
      if (a.fz.amax) {
        const float vk = (a.fz.p1 && v == 0.0f) ? 0.0f : v;
        const unsigned long long key = ((unsigned long long)fkey(vk) << 32) | (0xFFFFFFFFu - (uint32_t)lr);
        kbest = key > kbest ? key : kbest;
      }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < NR; i++) wc[i] = wn[i];
  }
}

// Weight-streaming int8 GEMV/skinny GEMM, persistent over output rows: each
// lane owns 32-byte sub-blocks of a weight row (the first rows loaded
// before the wait on the producing kernel, the next while the current
// compute), per-sub-block int32 sums by __dp4a, then the reference
// reduction per (output, token row) on separate lanes.  Compile-time
// variants keep each launched kernel small: RB bounds the token rows of
// the multi-row path (R <= RB); PRO adds the input-norm prologue (one
// WARPS-warp block per SM, so the prologue is paid once per SM); SINGLE is
// the one-row-per-step path for a second weight or more than 8 token rows.
template <int JM, int WARPS, int RB, bool PRO, bool SINGLE>
__global__ void __launch_bounds__(WARPS * 32) gemv_q8_kernel(const GemvArgs a) {
  constexpr int NR = gemv_nr<JM>();
  extern __shared__ __align__(16) float gsm[];
  // per-warp transposed product buffers (SINGLE: two of kGemvRB + 1 columns)
  constexpr int PW = (SINGLE ? 2 * (kGemvRB + 1) : RB * NR + 1) * JM * 32;
  float* P = gsm + (size_t)(threadIdx.x >> 5) * PW;
  float* P2 = P + (kGemvRB + 1) * JM * 32;
  float* pro = gsm + (size_t)WARPS * PW;
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * WARPS + (threadIdx.x >> 5);
  const int rb = a.gs >> 5, ng = a.K / a.gs;
  const int nstep = gridDim.x * WARPS;
  WRow<JM> w1, w2;
  WRow<JM> wc[NR];
  if (SINGLE) {
    const int rb2 = a.W2 ? a.gs2 >> 5 : 0, ng2 = a.W2 ? a.K2 / a.gs2 : 0;
    if (n0 < a.N) {
      load_wrow<JM>(w1, a.W + (size_t)n0 * a.K, a.ws + (size_t)n0 * ng, a.K, rb, lane);
      if (a.W2) load_wrow<JM>(w2, a.W2 + (size_t)n0 * a.K2, a.ws2 + (size_t)n0 * ng2, a.K2, rb2, lane);
    }
  } else {
#pragma unroll
    for (int i = 0; i < NR; i++) {
      const int r = n0 + i * nstep;
      if (r < a.N) load_wrow<JM>(wc[i], a.W + (size_t)r * a.K, a.ws + (size_t)r * ng, a.K, rb, lane);
    }
  }
  // the first step's row scales of the reducing lanes (one per row)
  float s_first = 0.0f, s2_first = 0.0f;
  if (SINGLE) {
    if (n0 < a.N && rb > 1 && ng == 1) s_first = __ldg(a.ws + n0);
    if (n0 < a.N && a.W2 && (a.gs2 >> 5) > 1 && a.K2 == a.gs2) s2_first = __ldg(a.ws2 + n0);
  } else {
    const int li = lane / a.R, lr = n0 + li * nstep;
    if (lane < NR * a.R && lr < a.N && rb > 1 && ng == 1) s_first = __ldg(a.ws + lr);
  }
  pdl_wait();
  if (!PRO) {
    unsigned long long kb = 0ull;
    if (SINGLE) gemv_rows<JM, WARPS, false>(a, a.xq, a.xs, w1, w2, P, P2, n0, lane, s_first, s2_first);
    else gemv_rows_multi<JM, WARPS, false, RB>(a, a.xq, a.xs, wc, P, n0, lane, s_first, kb);
    return;
  }
  // input-norm prologue: rows -> shared (every load issued before the
  // first store), one sequential sum of squares per row, then the (1+w)
  // scaling and per-32 quantisation (src/ops_norm.c:690-747,
  // src/ops_quant.c:2152-2282)
  const int warp = threadIdx.x >> 5;
  const int K = a.K, R = a.R, gpr = K / 32;
  float* fx = pro;                                   // [R][K]
  float* fw = fx + (size_t)R * K;                    // [K]
  int8_t* sxq = reinterpret_cast<int8_t*>(fw + K);   // [R][K]
  float* sxs = reinterpret_cast<float*>(sxq + (size_t)R * K);   // [R][K/32]
  float* sinv = sxs + (size_t)R * gpr;               // [R]
  {
    constexpr int U = 8;
    const int nv = (R * K + K) / 4, step = WARPS * 32;
    for (int i0 = threadIdx.x; i0 < nv; i0 += U * step) {
      float4 t[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int i = i0 + u * step;
        if (i < nv)
          t[u] = i * 4 < R * K ? __ldcg(reinterpret_cast<const float4*>(a.nx) + i)
                               : __ldg(reinterpret_cast<const float4*>(a.nw) + (i - R * K / 4));
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int i = i0 + u * step;
        if (i < nv) reinterpret_cast<float4*>(fx)[i] = t[u];
      }
    }
  }
  if (a.namax && blockIdx.x == 0 && threadIdx.x < R) a.namax[threadIdx.x] = 0ull;
  __syncthreads();
  if (R * 4 <= WARPS && K % 512 == 0 && R * (K + 16) <= WARPS * PW) {
    // four warps per row split the chain, the chain warps of rows 0-3 on
    // schedulers (0,1), (2,3), (0,1), (2,3); the squares go to the product
    // buffers, unused until the contraction
    __shared__ SplitSumShared split[WARPS / 4];
    if (warp < 4 * R) {
      const int r = warp >> 2, u = threadIdx.x - r * kSplitGroup, cw = 2 * (r & 1);
      const float ss = seq_sumsq_split(fx + (size_t)r * K, gsm + (size_t)r * (K + 16), K, u, cw, r, split[r]);
      if (u == 32 * cw) sinv[r] = rsqrt_body(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps));
    }
  } else {
    const int r = warp + WARPS * lane;
    if (r < R) sinv[r] = rsqrt_body(__fadd_rn(__fdiv_rn(seq_sumsq(fx + (size_t)r * K, K), (float)K), a.eps));
  }
  __syncthreads();
  const bool store = a.nout && blockIdx.x == 0;
  // one 32-group per warp step, row by row (no index division); a row's
  // groups of one warp are independent, so two of them overlap
  for (int r = 0; r < R; r++) {
    const float sr = sinv[r];
#pragma unroll 2
    for (int gg = warp; gg < gpr; gg += WARPS) {
      const int i = gg * 32 + lane;
      const float v = __fmul_rn(__fmul_rn(fx[(size_t)r * K + i], sr), __fadd_rn(1.0f, fw[i]));
      sxq[(size_t)r * K + i] = warp_quant32(v, &sxs[r * gpr + gg]);
      if (store) a.nout[(size_t)r * K + i] = v;
    }
  }
  __syncthreads();
  unsigned long long kb = 0ull;
  if (SINGLE) gemv_rows<JM, WARPS, true>(a, sxq, sxs, w1, w2, P, P2, n0, lane, s_first, s2_first);
  else gemv_rows_multi<JM, WARPS, true, RB>(a, sxq, sxs, wc, P, n0, lane, s_first, kb);
  if (!SINGLE && a.fz.amax) {
    // the block's arg-max per token row, one atomic per row
    __shared__ unsigned long long wbest[WARPS][kGemvRB];
    const int li = lane / R, lrr = lane - li * R;
    for (int rr = 0; rr < R; rr++) {
      const unsigned long long v = warp_max_u64((lane < NR * R && lrr == rr) ? kb : 0ull);
      if (lane == 0) wbest[warp][rr] = v;
    }
    __syncthreads();
    if (threadIdx.x < R) {
      unsigned long long m = 0ull;
      for (int w = 0; w < WARPS; w++) m = wbest[w][threadIdx.x] > m ? wbest[w][threadIdx.x] : m;
      atomicMax(a.fz.amax + threadIdx.x, m);
    }
    if (a.fz.sr) {
      // the last block: every row's arg-max is final, the hidden rows
      // (block 0's prologue) are written; the round's acceptance
      __shared__ int s_lastblk;
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) s_lastblk = atomicAdd(a.fz.counter, 1) == (int)gridDim.x - 1;
      __syncthreads();
      if (s_lastblk) {
        __threadfence();
        greedy_accept_all(a.fz);
        if (threadIdx.x == 0) *a.fz.counter = 0;
      }
    }
  }
}

// ------------------------------------------------------ tensor-core helpers

LZ_HD void mma_s8(int* d, const unsigned* a, unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// int32 -> float, exact for |v| < 2^22 (a 32-element int8 dot product is at
// most 32 * 127 * 127): the 1.5 * 2^23 magic add.
LZ_HD float i2f_small(int v) { return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f); }

// Per-element reduction state of one output element, the order of every
// float operation the reference's (q8_reduce): RB1 (gs = 32) keeps the four
// interleaved accumulators; otherwise a[0] is the running group dot and
// a[1] the sum over groups.
template <bool RB1>
struct RedState {
  float a[RB1 ? 4 : 2];
};

LZ_HD float mma_result(const RedState<false>& r) { return r.a[1]; }
LZ_HD float mma_result(const RedState<true>& r) {
  return __fadd_rn(__fadd_rn(r.a[0], r.a[2]), __fadd_rn(r.a[1], r.a[3]));
}

// ------------------------------------------- warp-tile tensor-core skinny GEMM
//
// For R > 8 token rows the weight-streaming GEMV would re-read every
// activation row per output row.  Here each 32-element sub-block dot
// product is one int8 tensor-core MMA (mma.sync m16n8k32, s8 x s8 -> s32,
// accumulator input zero): the exact int32 the reference accumulates per 32
// (src/ops_matmul.c:336-647); the reference's float epilogue
// (src/ops_epi.c:983-1023) then runs per (token, output) in K order in
// registers, so the kernel is bound by that float work, not by the MMA.
// One warp per 16 token rows x 8*NT outputs; no shared memory.  Each lane
// loads its MMA fragments straight from global memory: for sub-block s,
// lane (g, q) takes 8 contiguous bytes at s*32 + 8q of token rows g and
// g+8 (A) and of weight row g of each n tile (B), used as the fragment
// elements k = 4q..4q+3 and 16+4q..16+4q+3.  A and B share that byte
// permutation inside the sub-block, so each MMA (accumulator input zero)
// still yields the exact int32 sum over the 32 bytes.  With K never split
// across warps, each output's float reduction runs in K order in the
// lane that holds it.
// MT m tiles (A rows ra[i] for fragment rows g, rc[i] for rows g+8) by NT
// n tiles (weight rows nb[t] .. nb[t]+7, clamped to N-1).
template <int MT, int NT, bool RB1, int UF = 0>
LZ_HD void wmma_pass_mt(const int8_t* __restrict__ W, const float* __restrict__ ws, int N, int K, int gs,
                        const int8_t* __restrict__ xq, const float* __restrict__ xs, const int (&ra)[MT],
                        const int (&rc)[MT], const int (&nb)[NT], RedState<RB1> (&st)[MT][NT][4]) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int rb = gs >> 5, ng = K / gs, nsb = K >> 5;
  const int8_t* pa[MT];
  const int8_t* pc[MT];
  const float* xa[MT];
  const float* xc[MT];
#pragma unroll
  for (int i = 0; i < MT; i++) {
    pa[i] = xq + (size_t)ra[i] * K + tq * 8;
    pc[i] = xq + (size_t)rc[i] * K + tq * 8;
    xa[i] = xs + (size_t)ra[i] * nsb;
    xc[i] = xs + (size_t)rc[i] * nsb;
  }
  const int8_t* pb[NT];
  int oc[NT][2];
#pragma unroll
  for (int t = 0; t < NT; t++) {
    pb[t] = W + (size_t)min(nb[t] + gid, N - 1) * K + tq * 8;
    oc[t][0] = min(nb[t] + tq * 2, N - 1);
    oc[t][1] = min(nb[t] + tq * 2 + 1, N - 1);
  }
  float wrow[NT][2];
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int j = 0; j < 2; j++) wrow[t][j] = (!RB1 && ng == 1) ? __ldg(ws + oc[t][j]) : 0.0f;
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int e = 0; e < 4; e++)
#pragma unroll
        for (int j = 0; j < (RB1 ? 4 : 2); j++) st[i][t][e].a[j] = 0.0f;
  // fragments of U sub-blocks are loaded while the previous U compute
  constexpr int U = UF ? UF : (MT * 2 + NT >= 8 ? 1 : (MT * 2 + NT >= 5 ? 2 : 4));
  struct Frag {
    int2 A0[MT], A1[MT], B[NT];
    float x0[MT], x1[MT];
  };
  Frag cur[U], nxt[U];
  auto load = [&](Frag (&f)[U], int sb) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int s = sb + u;
      if (s < nsb) {
#pragma unroll
        for (int i = 0; i < MT; i++) {
          f[u].A0[i] = __ldg(reinterpret_cast<const int2*>(pa[i] + s * 32));
          f[u].A1[i] = __ldg(reinterpret_cast<const int2*>(pc[i] + s * 32));
          f[u].x0[i] = __ldg(xa[i] + s);
          f[u].x1[i] = __ldg(xc[i] + s);
        }
#pragma unroll
        for (int t = 0; t < NT; t++) f[u].B[t] = __ldg(reinterpret_cast<const int2*>(pb[t] + s * 32));
      }
    }
  };
  load(cur, 0);
  for (int sb = 0; sb < nsb; sb += U) {
    if (sb + U < nsb) load(nxt, sb + U);
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int s = sb + u;
      if (s >= nsb) break;
      const bool gend = !RB1 && (s + 1) % rb == 0;
      const int slot = s < (nsb & ~3) ? (s & 3) : 0;
#pragma unroll
      for (int t = 0; t < NT; t++) {
        float wg[2] = {wrow[t][0], wrow[t][1]};
        if (RB1) {
          wg[0] = __ldg(ws + (size_t)oc[t][0] * ng + s);
          wg[1] = __ldg(ws + (size_t)oc[t][1] * ng + s);
        } else if (gend && ng > 1) {
          wg[0] = __ldg(ws + (size_t)oc[t][0] * ng + s / rb);
          wg[1] = __ldg(ws + (size_t)oc[t][1] * ng + s / rb);
        }
#pragma unroll
        for (int i = 0; i < MT; i++) {
          const unsigned af[4] = {(unsigned)cur[u].A0[i].x, (unsigned)cur[u].A1[i].x, (unsigned)cur[u].A0[i].y,
                                  (unsigned)cur[u].A1[i].y};
          int d[4];
          mma_s8(d, af, (unsigned)cur[u].B[t].x, (unsigned)cur[u].B[t].y);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float a = i2f_small(d[e]);
            const float xsv = e < 2 ? cur[u].x0[i] : cur[u].x1[i];
            RedState<RB1>& R_ = st[i][t][e];
            if (!RB1) {
              R_.a[0] = __fadd_rn(R_.a[0], __fmul_rn(a, xsv));
              if (gend) {
                R_.a[1] = __fadd_rn(R_.a[1], __fmul_rn(R_.a[0], wg[e & 1]));
                R_.a[0] = 0.0f;
              }
            } else {
              const float p = __fmul_rn(a, __fmul_rn(xsv, wg[e & 1]));
#pragma unroll
              for (int j = 0; j < (RB1 ? 4 : 2); j++)
                if (j == slot) R_.a[j] = __fadd_rn(R_.a[j], p);
            }
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) cur[u] = nxt[u];
  }
}

// One m tile (the grouped expert kernels).
template <int NT, bool RB1>
LZ_HD void wmma_pass(const int8_t* __restrict__ W, const float* __restrict__ ws, int N, int K, int gs,
                     const int8_t* __restrict__ xq, const float* __restrict__ xs, int ra, int rc,
                     const int (&nb)[NT], RedState<RB1> (&st)[NT][4]) {
  const int rav[1] = {ra}, rcv[1] = {rc};
  wmma_pass_mt<1, NT, RB1>(W, ws, N, K, gs, xq, xs, rav, rcv, nb,
                           *reinterpret_cast<RedState<RB1>(*)[1][NT][4]>(&st));
}

// y (R x N, ld ldy) = [y +] W x (+ W2 x2) for R > 8 rows.  Warp tile 16 MT
// token rows x 8 NT outputs; block = 4 warps along N; grid
// (ceil(N / (32 NT)), ceil(R / (16 MT))).  Both weights of a dual call share
// the group-size class (the launcher checks).
template <int MT, int NT, bool RB1, int UF = 0>
__global__ void __launch_bounds__(128) gemm_q8_warp_kernel(const GemvArgs a) {
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int n0 = (blockIdx.x * 4 + warp) * 8 * NT, r0 = blockIdx.y * 16 * MT;
  // the weights do not depend on the producing kernel: the warp's rows of
  // both weights start streaming into L2 before the wait (once per n
  // range, by the first token tile's warps)
  if (n0 < a.N && blockIdx.y == 0 && lane == 0) {
    const int rows = min(8 * NT, a.N - n0);
    prefetch_l2(a.W + (size_t)n0 * a.K, (size_t)rows * a.K);
    prefetch_l2(a.ws + (size_t)n0 * (a.K / a.gs), (size_t)rows * (a.K / a.gs) * 4);
    if (a.W2) {
      prefetch_l2(a.W2 + (size_t)n0 * a.K2, (size_t)rows * a.K2);
      prefetch_l2(a.ws2 + (size_t)n0 * (a.K2 / a.gs2), (size_t)rows * (a.K2 / a.gs2) * 4);
    }
  }
  pdl_wait();
  if (n0 >= a.N) return;
  RedState<RB1> st[MT][NT][4];
  int nb[NT], ra[MT], rc[MT];
#pragma unroll
  for (int t = 0; t < NT; t++) nb[t] = n0 + t * 8;
#pragma unroll
  for (int i = 0; i < MT; i++) {
    ra[i] = min(r0 + i * 16 + gid, a.R - 1);
    rc[i] = min(r0 + i * 16 + gid + 8, a.R - 1);
  }
  wmma_pass_mt<MT, NT, RB1, UF>(a.W, a.ws, a.N, a.K, a.gs, a.xq, a.xs, ra, rc, nb, st);
  float v[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int e = 0; e < 4; e++) v[i][t][e] = mma_result(st[i][t][e]);
  if (a.W2) {
    wmma_pass_mt<MT, NT, RB1, UF>(a.W2, a.ws2, a.N, a.K2, a.gs2, a.xq2, a.xs2, ra, rc, nb, st);
#pragma unroll
    for (int i = 0; i < MT; i++)
#pragma unroll
      for (int t = 0; t < NT; t++)
#pragma unroll
        for (int e = 0; e < 4; e++) v[i][t][e] = __fadd_rn(v[i][t][e], mma_result(st[i][t][e]));
  }
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int r = r0 + i * 16 + gid + (e >= 2 ? 8 : 0);
        const int o = n0 + t * 8 + tq * 2 + (e & 1);
        if (r < a.R && o < a.N) {
          float* yp = a.y + (size_t)r * a.ldy + o;
          *yp = a.mode == 1 ? __fadd_rn(*yp, v[i][t][e]) : v[i][t][e];
        }
      }
}

// ------------------------------------------- TMA-staged tensor-core GEMM
//
// The same products and epilogue as gemm_q8_warp_kernel, with the operands
// staged in shared memory instead of loaded fragment by fragment from
// global memory (whose 8-row scattered loads kept the L1 pipe busy and the
// warps waiting).  A block of 8 consumer warps (2 along tokens x 4 along
// outputs, warp tile 16 MT x 8 NT) shares one token tile of 32 MT rows and
// one output tile of 32 NT rows; a producer warp streams 128-byte K slices
// of both (4 sub-blocks) with 2-D TMA loads into a ring of kTmaStages
// stages (128-byte swizzle, so the ldmatrix fragment reads are free of bank
// conflicts), with the per-32 activation scales (and, for gs = 32, the
// weight scales) as 16-byte boxes beside them.  Full / empty mbarriers pace
// the ring; every wait is bounded and a timeout sets *err and skips the
// stores.  Requires K (and K2) % 128 == 0.
constexpr int kTmaStages = 4;
constexpr int kTmaSub = 4;   // 32-byte sub-blocks per stage

struct alignas(64) GemmTmaArgs {
  CUtensorMap a, x, b, w;      // xq [rows][K] u8, xs [rows][K/32] f32, W [N][K] u8, ws [N][K/32] f32 (gs = 32)
  CUtensorMap a2, x2, b2, w2;  // second product over the same outputs
  const float* ws;             // weight scales, read directly when gs > 32
  const float* ws2;
  const int8_t* W;             // weight rows, for the L2 prefetch
  const int8_t* W2;
  float* y;
  int* err;
  int N, K, gs, K2, gs2, R, ldy, mode, dual;
};

LZ_HD float f4_at(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

template <int MT, int NT, bool RB1>
struct TmaTile {
  static constexpr int BM = 32 * MT, BN = 32 * NT;
  static constexpr int A = BM * 128, B = BN * 128, X = BM * 16, W = RB1 ? BN * 16 : 0;
  static constexpr int TILES = A + B;  // swizzled tiles of one stage (multiple of 1024 bytes)
  static constexpr int SMALL = X + W;  // scale boxes of one stage
  static constexpr size_t smem() { return 1024 + (size_t)kTmaStages * (TILES + SMALL) + 2 * kTmaStages * 8; }
};

// Consumer side of one product: pipeline iterations [itb, ite) (K slices
// c = it - itb) accumulated into st.  GM is the weight-scale class: 0 for
// gs = 32 (RB1), 1 for one group per row (gs = K), 2 for anything between.
// False on a barrier timeout.
template <int MT, int NT, bool RB1, int GM>
LZ_HD bool tma_pass(uint32_t base, const uint8_t* gsmall, uint32_t bars, int itb, int ite, int gs, int K,
                    const float* __restrict__ ws, int N, int n0, RedState<RB1> (&st)[MT][NT][4]) {
  using T = TmaTile<MT, NT, RB1>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int wm = warp >> 2, wn = warp & 3;
  const int rb = gs >> 5, ng = K / gs;
  int oc[NT][2];
  float wrow[NT][2];
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int j = 0; j < 2; j++) {
      oc[t][j] = min(n0 + wn * 8 * NT + t * 8 + tq * 2 + j, N - 1);
      wrow[t][j] = GM == 1 ? __ldg(ws + oc[t][j]) : 0.0f;
    }
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int e = 0; e < 4; e++)
#pragma unroll
        for (int j = 0; j < (RB1 ? 4 : 2); j++) st[i][t][e].a[j] = 0.0f;
  int gcnt = 0, gidx = 0;
  // lane addresses inside a stage (row & 7 == lane & 7 for every fragment row)
  const int sw = lane & 7;
  uint32_t aoff[MT];
#pragma unroll
  for (int i = 0; i < MT; i++) aoff[i] = (uint32_t)(wm * 16 * MT + i * 16 + sw + (((lane >> 3) & 1) << 3)) * 128u;
  const int ach = lane >> 4;
  const uint32_t boff = (uint32_t)T::A + (uint32_t)(wn * 8 * NT + (NT == 2 ? ((lane >> 4) << 3) : 0) + sw) * 128u;
  const int bch = (lane >> 3) & 1;
#pragma unroll 1
  for (int it = itb; it < ite; it++) {
    const int stg = it % kTmaStages;
    if (!mbar_wait(bars + 8 * stg, (it / kTmaStages) & 1)) return false;
    const uint32_t tile = base + stg * T::TILES;
    const float* xsm = reinterpret_cast<const float*>(gsmall + stg * T::SMALL);
    const float* wsm = xsm + T::BM * 4;
    // the stage's 4 sub-blocks: fragments and scales first, then the math
    unsigned bf[kTmaSub][NT][2], af[kTmaSub][MT][4];
    float4 xv[MT][2];
#pragma unroll
    for (int sl = 0; sl < kTmaSub; sl++) {
      if (NT == 2)
        ldsm_x4(tile + boff + ((uint32_t)((2 * sl + bch) ^ sw) << 4), bf[sl][0][0], bf[sl][0][1], bf[sl][NT - 1][0],
                bf[sl][NT - 1][1]);
      else
        ldsm_x2(tile + boff + ((uint32_t)((2 * sl + bch) ^ sw) << 4), bf[sl][0][0], bf[sl][0][1]);
#pragma unroll
      for (int i = 0; i < MT; i++)
        ldsm_x4(tile + aoff[i] + ((uint32_t)((2 * sl + ach) ^ sw) << 4), af[sl][i][0], af[sl][i][1], af[sl][i][2],
                af[sl][i][3]);
    }
#pragma unroll
    for (int i = 0; i < MT; i++) {
      const int rr = wm * 16 * MT + i * 16 + gid;
      xv[i][0] = *reinterpret_cast<const float4*>(xsm + rr * 4);
      xv[i][1] = *reinterpret_cast<const float4*>(xsm + (rr + 8) * 4);
    }
    float4 wv[NT][2];
    if (RB1) {
#pragma unroll
      for (int t = 0; t < NT; t++)
#pragma unroll
        for (int j = 0; j < 2; j++) wv[t][j] = *reinterpret_cast<const float4*>(wsm + (wn * 8 * NT + t * 8 + tq * 2 + j) * 4);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bars + 8 * (kTmaStages + stg));   // the stage is in registers: release it
#pragma unroll
    for (int sl = 0; sl < kTmaSub; sl++) {
      bool gend = false;
      float wg[NT][2];
      if (GM == 1) {
        gend = (it - itb) * kTmaSub + sl == (K >> 5) - 1;
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
          for (int j = 0; j < 2; j++) wg[t][j] = wrow[t][j];
      } else if (GM == 2) {
        gend = ++gcnt == rb;
        if (gend) {
          gcnt = 0;
#pragma unroll
          for (int t = 0; t < NT; t++)
#pragma unroll
            for (int j = 0; j < 2; j++) wg[t][j] = __ldg(ws + (size_t)oc[t][j] * ng + gidx);
          gidx++;
        }
      } else {
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
          for (int j = 0; j < 2; j++) wg[t][j] = f4_at(wv[t][j], sl);
      }
#pragma unroll
      for (int i = 0; i < MT; i++) {
        const float x0 = f4_at(xv[i][0], sl), x1 = f4_at(xv[i][1], sl);
#pragma unroll
        for (int t = 0; t < NT; t++) {
          int d[4];
          mma_s8(d, af[sl][i], bf[sl][t][0], bf[sl][t][1]);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float a = i2f_small(d[e]);
            const float xsv = e < 2 ? x0 : x1;
            RedState<RB1>& R_ = st[i][t][e];
            if (!RB1) {
              R_.a[0] = __fadd_rn(R_.a[0], __fmul_rn(a, xsv));
              if (gend) {
                R_.a[1] = __fadd_rn(R_.a[1], __fmul_rn(R_.a[0], wg[t][e & 1]));
                R_.a[0] = 0.0f;
              }
            } else {
              // K % 128 == 0: the interleaved accumulator of sub-block s is s & 3 == sl
              R_.a[sl] = __fadd_rn(R_.a[sl], __fmul_rn(a, __fmul_rn(xsv, wg[t][e & 1])));
            }
          }
        }
      }
    }
  }
  return true;
}

template <int MT, int NT, bool RB1, int GM>
__global__ void __launch_bounds__(288) gemm_q8_tma_kernel(const __grid_constant__ GemmTmaArgs p) {
  using T = TmaTile<MT, NT, RB1>;
  extern __shared__ uint8_t tma_smem[];
  const uint32_t raw = smem_u32(tma_smem);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t small = base + kTmaStages * T::TILES;
  const uint32_t bars = small + kTmaStages * T::SMALL;  // full[s] at +8s, empty[s] at +8(kTmaStages + s)
  const uint8_t* gsmall = tma_smem + (small - raw);
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * T::BN, r0 = blockIdx.y * T::BM;
  const int nsb = p.K >> 5, nsb2 = p.dual ? p.K2 >> 5 : 0;
  const int it1 = (nsb + kTmaSub - 1) / kTmaSub, nit = it1 + (nsb2 + kTmaSub - 1) / kTmaSub;
  if (warp == 8 && lane == 0 && blockIdx.y == 0) {  // weights stream into L2 before the wait
    const int rows = min(T::BN, p.N - n0);
    prefetch_l2(p.W + (size_t)n0 * p.K, (size_t)rows * p.K);
    if (p.dual) prefetch_l2(p.W2 + (size_t)n0 * p.K2, (size_t)rows * p.K2);
  }
  pdl_wait();
  if (threadIdx.x == 256) {
    for (int s = 0; s < kTmaStages; s++) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (kTmaStages + s), 8);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 8) {
    if (lane != 0) return;
    bool ok = true;
    int it = 0;
    const bool skip0 = g_dbg_skip_stage != 0;   // test hook: stage 0 is never filled
    for (; it < nit; it++) {
      const int stg = it % kTmaStages;
      if (it >= kTmaStages && !mbar_wait(bars + 8 * (kTmaStages + stg), (it / kTmaStages - 1) & 1)) {
        ok = false;
        break;
      }
      fence_proxy_async_smem();
      if (skip0 && it == 0) continue;
      const bool two = it >= it1;
      const int c = two ? it - it1 : it;
      const uint32_t full = bars + 8 * stg, tile = base + stg * T::TILES, sm = small + stg * T::SMALL;
      mbar_expect_tx(full, T::A + T::B + T::X + T::W);
      tma_load_2d(tile, two ? &p.a2 : &p.a, c * 128, r0, full);
      tma_load_2d(tile + T::A, two ? &p.b2 : &p.b, c * 128, n0, full);
      tma_load_2d(sm, two ? &p.x2 : &p.x, c * kTmaSub, r0, full);
      if (RB1) tma_load_2d(sm + T::X, two ? &p.w2 : &p.w, c * kTmaSub, n0, full);
    }
    if (!ok) atomicExch(p.err, 1);
    // every copy issued lands before the block exits
    for (int j = max(0, it - kTmaStages); j < it; j++) mbar_wait(bars + 8 * (j % kTmaStages), (j / kTmaStages) & 1);
    return;
  }
  RedState<RB1> st[MT][NT][4];
  float v[MT][NT][4];
  bool ok = tma_pass<MT, NT, RB1, GM>(base, gsmall, bars, 0, it1, p.gs, p.K, p.ws, p.N, n0, st);
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int e = 0; e < 4; e++) v[i][t][e] = mma_result(st[i][t][e]);
  if (ok && p.dual) {
    ok = tma_pass<MT, NT, RB1, GM>(base, gsmall, bars, it1, nit, p.gs2, p.K2, p.ws2, p.N, n0, st);
#pragma unroll
    for (int i = 0; i < MT; i++)
#pragma unroll
      for (int t = 0; t < NT; t++)
#pragma unroll
        for (int e = 0; e < 4; e++) v[i][t][e] = __fadd_rn(v[i][t][e], mma_result(st[i][t][e]));
  }
  if (!ok) {
    atomicExch(p.err, 1);
    return;
  }
  const int wm = warp >> 2, wn = warp & 3, gid = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int i = 0; i < MT; i++)
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int r = r0 + wm * 16 * MT + i * 16 + gid + (e >= 2 ? 8 : 0);
        const int o = n0 + wn * 8 * NT + t * 8 + tq * 2 + (e & 1);
        if (r < p.R && o < p.N) {
          float* yp = p.y + (size_t)r * p.ldy + o;
          *yp = p.mode == 1 ? __fadd_rn(*yp, v[i][t][e]) : v[i][t][e];
        }
      }
}

// Test hook: one thread waits on an mbarrier that nothing ever arrives on.
// The bounded wait gives up after about a second and the kernel reports
// through *err, with no fault and the context still usable.
__global__ void wait_timeout_probe_kernel(int* err) {
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x == 0) {
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    mbar_fence_init();
    if (!mbar_wait(b, 0)) atomicExch(err, 2);
  }
}

// --------------------------------------------------------- row kernels

// rmsnorm (1+w) of one row, then per-32 quantisation of the result; the
// float result is stored too when `out` is non-null; `amax_clear`, when
// non-null, zeroes this row's arg-max slot for a following lm_head.
// One block per row.  src/ops_norm.c:690-747, src/ops_quant.c:2152-2282.
__global__ void rmsnorm_quant_kernel(const float* __restrict__ x, int ldx,
                                     const float* __restrict__ w, int n, float eps,
                                     float* out, int ldo, int8_t* xq, float* xs,
                                     unsigned long long* amax_clear) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float sm[];
  __shared__ float s_inv;
  const int r = blockIdx.x;
  const float* xr = x + (size_t)r * ldx;
  // each thread's loads issued together, then its stores
  for (int i0 = threadIdx.x; i0 < n; i0 += kRowLoadU * blockDim.x) {
    float a[kRowLoadU], b[kRowLoadU];
#pragma unroll
    for (int u = 0; u < kRowLoadU; u++) {
      const int i = i0 + u * blockDim.x;
      a[u] = i < n ? xr[i] : 0.0f;
      b[u] = i < n ? __ldg(w + i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kRowLoadU; u++) {
      const int i = i0 + u * blockDim.x;
      if (i < n) {
        sm[i] = a[u];
        sm[n + i] = b[u];
      }
    }
  }
  if (amax_clear && threadIdx.x == 0) amax_clear[r] = 0ull;
  __syncthreads();
  if (n % 512 == 0 && blockDim.x >= kSplitGroup) {
    // the first four warps split the chain, squares into sm[2n..3n+16)
    __shared__ SplitSumShared split;
    if (threadIdx.x < kSplitGroup) {
      const float ss = seq_sumsq_split(sm, sm + 2 * (size_t)n, n, threadIdx.x, 0, 0, split);
      if (threadIdx.x == 0) s_inv = rsqrt_body(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
    }
  } else if (threadIdx.x == 0) {
    s_inv = rsqrt_body(__fadd_rn(__fdiv_rn(seq_sumsq(sm, n), (float)n), eps));
  }
  __syncthreads();
  const float inv = s_inv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  // a warp's groups are independent: four in flight
#pragma unroll 4
  for (int g = warp; g < n / 32; g += nw) {
    const int i = g * 32 + lane;
    const float o = __fmul_rn(__fmul_rn(sm[i], inv), __fadd_rn(1.0f, sm[n + i]));
    if (out) out[(size_t)r * ldo + i] = o;
    xq[(size_t)r * n + i] = warp_quant32(o, &xs[(size_t)r * (n / 32) + g]);
  }
}

// Embedding rows: x[i] = q[i] * scale[group]  (src/ops_epi.c:1276-1280).
__global__ void embed_kernel(const int8_t* __restrict__ eq, const float* __restrict__ es,
                             int gs, int d, const int* __restrict__ tok, float* x) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const size_t base = (size_t)tok[r] * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    x[(size_t)r * d + i] = __fmul_rn((float)eq[base + i], es[(base + i) / gs]);
}

// silu(gate)*up then per-32 quantisation (src/forward_kda.c:1082-1085
// followed by lz_quantize_q8).  gate at column g0, up at column u0.
__global__ void swiglu_quant_kernel(const float* __restrict__ src, int lds, int g0, int u0,
                                    int n, int8_t* xq, float* xs) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* row = src + (size_t)r * lds;
  // four of a warp's groups at a time, their loads issued together
  constexpr int U = 4;
  const int ng = n / 32;
  for (int gb = warp; gb < ng; gb += U * nw) {
    float gv[U], uv[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = (gb + u * nw) * 32 + lane;
      gv[u] = gb + u * nw < ng ? row[g0 + i] : 0.0f;
      uv[u] = gb + u * nw < ng ? row[u0 + i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int g = gb + u * nw;
      if (g < ng) {
        const float a = __fmul_rn(silu(gv[u]), uv[u]);
        xq[(size_t)r * n + g * 32 + lane] = warp_quant32(a, &xs[(size_t)r * ng + g]);
      }
    }
  }
}

// Arg-max of each row, first index on ties, into a packed 64-bit slot
// (key << 32 | ~index) combined across blocks by atomicMax; the slot must
// be zero beforehand.  p1_mode = 0 compares by the total key of
// src/sampler.c:224-240; p1_mode = 1 by float `>` (lz_argmax_p1,
// src/sampler.c:279-295), so -0 and +0 compare equal.
constexpr int kArgmaxChunk = 4096;
__global__ void argmax_kernel(const float* __restrict__ logits, int V, int p1_mode,
                              unsigned long long* slot) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.y;
  const float* row = logits + (size_t)r * V;
  const int i0 = blockIdx.x * kArgmaxChunk, i1 = min(V, i0 + kArgmaxChunk);
  unsigned long long best = 0ull;
#pragma unroll 4
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float v = __ldg(row + i);
    if (p1_mode && v == 0.0f) v = 0.0f;
    const unsigned long long key = ((unsigned long long)fkey(v) << 32) | (0xFFFFFFFFu - (uint32_t)i);
    best = key > best ? key : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) atomicMax(slot + r, best);
}

LZ_HD int argmax_index(unsigned long long packed) { return (int)(0xFFFFFFFFu - (uint32_t)packed); }

// ---------------------------------------------------------------- KDA

struct KdaSeq {            // one sequence's rows inside a forward batch
  int row0, nrows, base_slot, seq;
};

// Arguments of the KDA layer kernel (one layer, every sequence of the
// forward batch).
struct KdaArgs {
  const float* inproj; int ldi;            // [R][n_in]: q | k | v | g | f_a | b (the fused in-projection)
  int kdim, off_g, off_fa, off_b, rank;
  const float* cw;                         // conv1d weights [conv_dim][4]
  float* conv_state;                       // this layer's [conv_dim][3] of ring slot 0, sequence 0
  size_t conv_seq_stride, conv_slot_stride;
  const int8_t* fbq; const float* fbs; int fb_gs;   // f_b [nv 64][rank] Q8_0
  const float* a_log; const float* dt_bias; float lb;
  const KdaSeq* seqs;
  int8_t* st_hi; int8_t* st_lo; float* st_sc;       // two-plane state ring
  size_t seq_stride_q, slot_stride_q; int layer_off_q;
  int depth, adv; float ssm_scale;
  const float* o_norm; float eps; int vdim;
  int8_t* oq; float* os;                   // quantised gated-norm output [R][vdim]
};

// The KDA layer of one (sequence, head): the short conv1d of the head's 192
// channels (q, k, v) with the conv ring history (src/ops_conv1d.c:26-60),
// the decay gate of its 64 keys from the f_b projection
// (src/forward_kda.c:277-404), then the recurrence with the 64x64 two-plane
// int8 state resident in shared memory.  Everything that does not read the
// state runs for a batch of up to kRecurTB tokens at once: the conv (one
// thread per channel, tokens in order, the history in registers), the f_a
// quantisation and the gate, l2norm(q) * kd^-1/2, l2norm(k), beta =
// sigmoid(b), and the products k*g and q*g; then per token, serially,
// pass 1 (u = S^T(g.k) and w = S^T(g.q), each a sequential sum over the 64
// state rows on its own thread per value column, the scale product sc *
// (k*g) formed in place; k.q on another thread), u = (v - u)*beta, and
// pass 2 (each state row g*S + k*u requantised in two planes, four 32-wide
// groups per warp at a time, the head output w + u*kq beside it);
// finally the gated RMSNorm and per-32 quantisation of every token's
// output.  src/forward_kda.c:856-936 and 1029-1040, src/ops_gdn.c:2488-2778,
// src/ops_gdn.c:1191-1340, src/ops_norm.c:749-842.
//
// SPLIT = 2 runs a head as a cluster of two CTAs, one per 32-wide value
// group: the state columns (and their row scales) of the two groups never
// meet in the recurrence - pass 1 sums down a column, pass 2 requantises a
// (row, group) - so each CTA holds and updates only its half; the
// per-key work (conv, gate, norms) is done by both.  The gated RMSNorm
// needs the whole head output: each CTA writes its 32 columns into the
// peer's shared memory, then one cluster barrier.  SPLIT = 1 is one CTA
// per head.
constexpr int kRecurThreads = 256;
constexpr int kRecurTB = 4;
constexpr int kRankMax = 128;

// One two-plane requantisation of a 32-wide state group held one element
// per lane (src/ops_gdn.c:1191-1340): hi = q8 of buf, residual rounded
// half up into hi when possible, lo = rne(residual * 256).
// Also returns e = hi + lo / 256, the element as the next token dequantises
// it (hi as a float is exact, so it is adjusted with hq).
LZ_HD void requant_2p(float buf, float iv, int8_t& h8, int8_t& l8, float& e) {
  const float f = __fmul_rn(buf, iv);
  const int hq0 = q8_clamp(q8_round(f));
  const float hf0 = (float)hq0;
  const float res0 = __fsub_rn(f, hf0);
  // the residual's half-up correction, by selects (the two cases exclude
  // each other)
  const bool up = res0 >= 0.5f && hq0 < 127, dn = res0 < -0.5f && hq0 > -127;
  const int hq = hq0 + (up ? 1 : 0) - (dn ? 1 : 0);
  const float hf = up ? __fadd_rn(hf0, 1.0f) : (dn ? __fsub_rn(hf0, 1.0f) : hf0);
  const float res = up ? __fsub_rn(res0, 1.0f) : (dn ? __fadd_rn(res0, 1.0f) : res0);
  h8 = (int8_t)hq;
  const int lq = q8_clamp(q8_round(__fmul_rn(res, kLoScale)));
  l8 = (int8_t)lq;
  e = __fadd_rn(hf, __fmul_rn((float)lq, 1.0f / kLoScale));
}

template <int NTH, int SPLIT>
LZ_HD void kda_layer(const KdaArgs& a) {
  pdl_trigger();
  constexpr int KD = 64, VD = 64, VC = VD / SPLIT, GPC = VC / 32, TB = kRecurTB, NW = NTH / 32;
  static_assert(NTH >= 3 * KD && NTH >= TB * KD && NTH >= 2 * VC + TB, "thread roles");
  static_assert(2 * NW >= 3 * TB, "norm chains per batch exceed the warps");
  // f_a groups a warp stages, and the (g | b) values a thread stages
  constexpr int FG = (TB * kRankMax / 32 + NW - 1) / NW;
  constexpr int MI = (TB * (VC + 1) + NTH - 1) / NTH;
  __shared__ __align__(16) int8_t hi[KD][VC];
  __shared__ __align__(16) int8_t lo[KD][VC];
  // the state dequantised (hi + lo / 256, unscaled), refreshed right after
  // each requantisation
  __shared__ __align__(16) float E[KD][VC];
  __shared__ float sc[KD][GPC];
  __shared__ __align__(16) float qn[TB][KD], kn[TB][KD], gv[TB][KD], KG[TB][KD], QG[TB][KD];
  // the current token's scale products sc * (k*g) and sc * (q*g) of pass 1
  __shared__ float SCK[KD][GPC], SCQ[KD][GPC];
  __shared__ __align__(16) float vcs[TB][VC], zs[TB][VC];
  // the head outputs of a batch, both value groups (SPLIT = 2: the peer
  // writes its group into this copy); two buffers by batch parity, so a
  // peer one batch ahead never writes the buffer this CTA still reads
  __shared__ __align__(16) float OUT2[2][TB][VD];
  __shared__ __align__(16) float U[VC], AW[VC];
  __shared__ float inv_q[TB], inv_k[TB], beta[TB], braw[TB], kqs[TB], inv_o[TB];
  __shared__ __align__(16) int8_t LQ[TB][kRankMax];
  __shared__ float LS[TB][kRankMax / 32];
  // this head's f_b rows and their scales
  __shared__ __align__(16) int8_t FB[KD][kRankMax];
  __shared__ float FBS[KD][kRankMax / 32];
  const int h = blockIdx.x / SPLIT, grp = SPLIT == 1 ? 0 : (int)(blockIdx.x % SPLIT), vcol0 = grp * VC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nsb = a.rank / 32, rbf = a.fb_gs / 32, ngf = a.rank / a.fb_gs;
  // weights do not change during a round: loaded before the wait on the
  // producing kernel
  for (int q = tid; q < KD * nsb * 2; q += NTH) {
    const int j = q / (nsb * 2), c16 = q - j * nsb * 2;
    reinterpret_cast<int4*>(&FB[j][0])[c16] =
        __ldg(reinterpret_cast<const int4*>(a.fbq + (size_t)(h * KD + j) * a.rank) + c16);
  }
  for (int q = tid; q < KD * ngf; q += NTH) {
    const int j = q / ngf, u = q - j * ngf;
    FBS[j][u] = __ldg(a.fbs + (size_t)(h * KD + j) * ngf + u);
  }
  const float decay = exp_body(__ldg(a.a_log + h));   // exp(A_log) of the head (src/forward_kda.c:277-404)
  const float dtb = __ldg(a.dt_bias + h * KD + (tid & 63));
  const int part = tid >> 6, ci = tid & 63;            // conv channel of threads 0..191: q, k, v of this head
  const int chan = part == 0 ? h * KD + ci : part == 1 ? a.kdim + h * KD + ci : 2 * a.kdim + h * VD + ci;
  float4 cwv = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid < 3 * KD) cwv = __ldg(reinterpret_cast<const float4*>(a.cw) + chan);
  pdl_wait();
  const KdaSeq sq = a.seqs[blockIdx.y];
  const size_t head_off = (size_t)a.layer_off_q + (size_t)h * KD * VD;
  const size_t seq_off = (size_t)sq.seq * a.seq_stride_q;
  float* cst0 = a.conv_state + (size_t)sq.seq * a.conv_seq_stride + (size_t)chan * 3;
  // a batch's rows, every load issued before the first store: the conv
  // inputs of this thread's channel, whole 32-wide f_a groups per warp
  // (quantised from registers), and the z (gate) and b values
  float xr[TB], fa[FG], mi[MI];
  auto issue = [&](int t0, int nt) {
    if (tid < 3 * KD) {
#pragma unroll
      for (int t = 0; t < TB; t++)
        if (t < nt) xr[t] = a.inproj[(size_t)(sq.row0 + t0 + t) * a.ldi + chan];
    }
#pragma unroll
    for (int i = 0; i < FG; i++) {
      const int g = NW - 1 - warp + i * NW;
      if (g < nt * nsb) {
        const int t = g / nsb, gg = g - t * nsb;
        fa[i] = a.inproj[(size_t)(sq.row0 + t0 + t) * a.ldi + a.off_fa + gg * 32 + lane];
      }
    }
#pragma unroll
    for (int i = 0; i < MI; i++) {
      const int q = tid + i * NTH;
      if (q < nt * VC) {
        const int t = q / VC, c = q - t * VC;
        mi[i] = a.inproj[(size_t)(sq.row0 + t0 + t) * a.ldi + a.off_g + h * VD + vcol0 + c];
      } else if (q < nt * VC + nt) {
        mi[i] = a.inproj[(size_t)(sq.row0 + t0 + q - nt * VC) * a.ldi + a.off_b + h];
      }
    }
  };
  // the state of this CTA's columns and the conv history, in flight with
  // the first batch's rows
  constexpr int SQ = KD * VC / 16;       // 16-byte pieces per plane
  int4 sh = make_int4(0, 0, 0, 0), sl = sh;
  float ssc = 0.0f, c0 = 0.0f, c1 = 0.0f, c2 = 0.0f;
  {
    const size_t off = seq_off + (size_t)sq.base_slot * a.slot_stride_q + head_off;
    if (tid < SQ) {
      const int row = tid / (VC / 16), c16 = tid - row * (VC / 16);
      const size_t o = off + (size_t)row * VD + vcol0 + c16 * 16;
      sh = *reinterpret_cast<const int4*>(a.st_hi + o);
      sl = *reinterpret_cast<const int4*>(a.st_lo + o);
    }
    if (tid < KD * GPC) ssc = a.st_sc[off / 32 + (tid / GPC) * (VD / 32) + grp * GPC + tid % GPC];
    if (tid < 3 * KD) {
      const float* st = cst0 + (size_t)sq.base_slot * a.conv_slot_stride;
      c0 = st[0]; c1 = st[1]; c2 = st[2];
    }
  }
  issue(0, min(TB, sq.nrows));
  if (tid < SQ) {
    const int row = tid / (VC / 16), c16 = tid - row * (VC / 16);
    *reinterpret_cast<int4*>(&hi[row][c16 * 16]) = sh;
    *reinterpret_cast<int4*>(&lo[row][c16 * 16]) = sl;
    const int8_t* hb = reinterpret_cast<const int8_t*>(&sh);
    const int8_t* lb = reinterpret_cast<const int8_t*>(&sl);
#pragma unroll
    for (int j = 0; j < 16; j++)
      E[row][c16 * 16 + j] = __fadd_rn((float)hb[j], __fmul_rn((float)lb[j], 1.0f / kLoScale));
  }
  if (tid < KD * GPC) sc[tid / GPC][tid % GPC] = ssc;
  int t0 = 0;
  // ring slot of batch token t (verify steps): this CTA's state planes and
  // row scales, copied from shared memory in 16-byte pieces by threads
  // i0, i0 + step, ...
  auto ring_copy = [&](int t, int i0, int step) {
    const size_t ring = seq_off + (size_t)((sq.base_slot + t0 + t + 1) % a.depth) * a.slot_stride_q + head_off;
    for (int q = i0; q < 2 * SQ + KD * GPC; q += step) {
      if (q < 2 * SQ) {
        const int pl = q / SQ, qq = q - pl * SQ, row = qq / (VC / 16), c16 = qq - row * (VC / 16);
        const size_t o = ring + (size_t)row * VD + vcol0 + c16 * 16;
        if (pl == 0) *reinterpret_cast<int4*>(a.st_hi + o) = *reinterpret_cast<const int4*>(&hi[row][c16 * 16]);
        else *reinterpret_cast<int4*>(a.st_lo + o) = *reinterpret_cast<const int4*>(&lo[row][c16 * 16]);
      } else {
        const int u = q - 2 * SQ, kk = u / GPC, gl = u - kk * GPC;
        a.st_sc[ring / 32 + kk * (VD / 32) + grp * GPC + gl] = sc[kk][gl];
      }
    }
  };
  for (; t0 < sq.nrows; t0 += TB) {
    const int nt = min(TB, sq.nrows - t0);
    float (*OUT)[VD] = OUT2[(t0 / TB) & 1];
    if (t0 > 0) issue(t0, nt);
#pragma unroll
    for (int i = 0; i < MI; i++) {
      const int q = tid + i * NTH;
      if (q < nt * VC) zs[q / VC][q % VC] = mi[i];
      else if (q < nt * VC + nt) braw[q - nt * VC] = mi[i];
    }
    // the conv1d of the batch (src/ops_conv1d.c:26-60), then SiLU
    if (tid < 3 * KD) {
      // unrolled over the batch: the tokens' convolutions read only the raw
      // inputs and the shifted history, so their SiLUs overlap
#pragma unroll
      for (int t = 0; t < TB; t++) {
        if (t >= nt) break;
        const float xv = xr[t];
        float sum = 0.0f;
        sum = __fadd_rn(sum, __fmul_rn(cwv.x, c0));
        sum = __fadd_rn(sum, __fmul_rn(cwv.y, c1));
        sum = __fadd_rn(sum, __fmul_rn(cwv.z, c2));
        sum = __fadd_rn(sum, __fmul_rn(cwv.w, xv));
        const float y = silu(sum);
        if (part == 0) qn[t][ci] = y;
        else if (part == 1) kn[t][ci] = y;
        else if (ci >= vcol0 && ci < vcol0 + VC) vcs[t][ci - vcol0] = y;
        c0 = c1; c1 = c2; c2 = xv;
        if (a.adv && grp == 0) {
          float* d = cst0 + (size_t)((sq.base_slot + t0 + t + 1) % a.depth) * a.conv_slot_stride;
          d[0] = c0; d[1] = c1; d[2] = c2;
        }
      }
    }
    // the f_a rows quantised per 32 (src/ops_quant.c:2152-2282)
#pragma unroll
    for (int i = 0; i < FG; i++) {
      const int g = NW - 1 - warp + i * NW;
      if (g < nt * nsb) {
        const int t = g / nsb, gg = g - t * nsb;
        LQ[t][gg * 32 + lane] = warp_quant32(fa[i], &LS[t][gg]);
      }
    }
    __syncthreads();
    // the decay gate of this head's 64 keys: exp(lb sigmoid(exp(A) (f_b(f_a) + dt)))
    if (tid < nt * KD) {
      const int t = tid >> 6, jj = tid & 63;
      const float* wsr = FBS[jj];
      __align__(16) float p[kRankMax / 32];
#pragma unroll
      for (int u = 0; u < kRankMax / 32; u++)
        if (u < nsb) {
          const int4 wa = *reinterpret_cast<const int4*>(&FB[jj][u * 32]);
          const int4 wb = *reinterpret_cast<const int4*>(&FB[jj][u * 32 + 16]);
          const int4 xa = *reinterpret_cast<const int4*>(&LQ[t][u * 32]);
          const int4 xb = *reinterpret_cast<const int4*>(&LQ[t][u * 32 + 16]);
          const float av = (float)dot32(wa, wb, xa, xb);
          p[u] = rbf > 1 ? __fmul_rn(av, LS[t][u]) : __fmul_rn(av, __fmul_rn(LS[t][u], wsr[u]));
        }
      const float pre = __fadd_rn(q8_reduce(p, wsr, rbf, ngf), dtb);
      const float gg = __fmul_rn(a.lb, sigmoid(__fmul_rn(decay, pre)));
      gv[t][jj] = exp_body(gg);
    }
    {                                          // 3 nt independent chains, two per warp, after the gate's warps
      const int c = ((warp + NW - 2 * nt) % NW) * 2 + (lane >> 4);
      if ((lane & 15) == 0 && c < 3 * nt) {
        const int t = c % nt, which = c / nt;
        if (which == 0) inv_q[t] = rsqrt_body(__fadd_rn(seq_sumsq(qn[t], KD), kL2Eps));
        else if (which == 1) inv_k[t] = rsqrt_body(__fadd_rn(seq_sumsq(kn[t], KD), kL2Eps));
        else beta[t] = sigmoid(braw[t]);
      }
    }
    __syncthreads();
    for (int q = tid; q < nt * KD; q += NTH) {
      const int t = q >> 6, i = q & 63;
      const float qv = __fmul_rn(__fmul_rn(qn[t][i], inv_q[t]), a.ssm_scale);
      const float kv = __fmul_rn(kn[t][i], inv_k[t]);
      qn[t][i] = qv;
      kn[t][i] = kv;
      KG[t][i] = __fmul_rn(kv, gv[t][i]);
      QG[t][i] = __fmul_rn(qv, gv[t][i]);
      if (t == 0)
#pragma unroll
        for (int gl = 0; gl < GPC; gl++) {
          SCK[i][gl] = __fmul_rn(sc[i][gl], KG[0][i]);
          SCQ[i][gl] = __fmul_rn(sc[i][gl], QG[0][i]);
        }
    }
    __syncthreads();
    for (int t = 0; t < nt; t++) {
      // pass 1: one sequential chain over the 64 state rows per thread, in
      // the reference's order: u = S^T (g.k) on threads c < VC, w = S^T
      // (g.q) on threads VC + c; u = (v - u) * beta.  The batch's k.q
      // chains run beside the first token's.
      if (tid < 2 * VC) {
        const bool isw = tid >= VC;
        const int c = isw ? tid - VC : tid, gl = c >> 5;
        const float* Sx = isw ? &SCQ[0][gl] : &SCK[0][gl];
        float acc = 0.0f;
        // 16 products formed ahead of their adds (the adds stay in order)
#pragma unroll
        for (int k0 = 0; k0 < KD; k0 += 16) {
          float pr[16];
#pragma unroll
          for (int j = 0; j < 16; j++) pr[j] = __fmul_rn(E[k0 + j][c], Sx[(k0 + j) * GPC]);
#pragma unroll
          for (int j = 0; j < 16; j++) acc = __fadd_rn(acc, pr[j]);
        }
        if (isw) AW[c] = acc;
        else U[c] = __fmul_rn(__fsub_rn(vcs[t][c], acc), beta[t]);
      } else if (t == 0 && tid < 2 * VC + nt) {
        const int tt = tid - 2 * VC;
        float kq = 0.0f;
#pragma unroll 8
        for (int kk = 0; kk < KD; kk++) kq = __fadd_rn(kq, __fmul_rn(kn[tt][kk], qn[tt][kk]));
        kqs[tt] = kq;
      } else if (a.adv && t > 0 && tid >= 2 * VC + TB) {
        // the previous token's ring slot, from the shared state, by the
        // threads pass 1 leaves idle
        ring_copy(t - 1, tid - (2 * VC + TB), NTH - (2 * VC + TB));
      }
      __syncthreads();
      // the head output w + u * kq of this CTA's columns
      if (tid < VC) OUT[t][vcol0 + tid] = __fadd_rn(AW[tid], __fmul_rn(U[tid], kqs[t]));
      // pass 2: the (state row, 32-wide group) units, four per warp at a
      // time with their max reductions interleaved; the new row scales
      // also give the next token's pass-1 products
      for (int u0 = warp * 4; u0 < KD * GPC; u0 += NW * 4) {
        float buf[4];
        uint32_t am[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int unit = u0 + c, kk = unit / GPC, gl = unit % GPC, col = gl * 32 + lane;
          const float scg = __fmul_rn(sc[kk][gl], gv[t][kk]);   // sc * g, before this unit's scale is replaced
          buf[c] = __fadd_rn(__fmul_rn(E[kk][col], scg), __fmul_rn(kn[t][kk], U[col]));
          am[c] = abs_bits(buf[c]);
        }
#pragma unroll
        for (int c = 0; c < 4; c++) am[c] = __reduce_max_sync(0xffffffffu, am[c]);
        // the four groups' scales on lanes 0-3 at once, then broadcast
        float sg4, iv4;
        q8_scale_from_amax(lane == 1 ? am[1] : lane == 2 ? am[2] : lane == 3 ? am[3] : am[0], &sg4, &iv4);
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int unit = u0 + c, kk = unit / GPC, gl = unit % GPC, col = gl * 32 + lane;
          const float sg = __shfl_sync(0xffffffffu, sg4, c), iv = __shfl_sync(0xffffffffu, iv4, c);
          int8_t h8, l8;
          float e;
          requant_2p(buf[c], iv, h8, l8, e);
          E[kk][col] = e;
          hi[kk][col] = h8;
          lo[kk][col] = l8;
          if (lane == 0) {
            sc[kk][gl] = sg;
            if (t + 1 < nt) {
              SCK[kk][gl] = __fmul_rn(sg, KG[t + 1][kk]);
              SCQ[kk][gl] = __fmul_rn(sg, QG[t + 1][kk]);
            }
          }
        }
      }
      __syncthreads();
    }
    // the batch's last ring slot
    if (a.adv) ring_copy(nt - 1, tid, NTH);
    // this CTA's half of every token's head output into the peer's copy,
    // then one cluster barrier: both copies whole
    if (SPLIT > 1) {
      for (int q = tid; q < nt * VC; q += NTH) {
        const int t = q / VC, c = q - t * VC;
        st_peer_f32(&OUT[t][vcol0 + c], (uint32_t)(grp ^ 1), OUT[t][vcol0 + c]);
      }
      cluster_barrier();
    }
    // gated RMSNorm of every token's head output, then per-32 quantisation;
    // each thread's first output's norm weight and gate are formed while
    // the sums of squares run
    float pw = 0.0f, pz = 0.0f;
    if (tid < nt * VC) {
      const int t = tid / VC, c = tid - t * VC;
      pw = a.o_norm[vcol0 + c];
      pz = silu(zs[t][c]);
    }
    if (lane == 0 && warp < nt)
      inv_o[warp] = rsqrt_body(__fadd_rn(__fdiv_rn(seq_sumsq(OUT[warp], VD), (float)VD), a.eps));
    __syncthreads();
    for (int q = tid; q < nt * VC; q += NTH) {
      const int t = q / VC, c = q - t * VC, i = vcol0 + c;
      const size_t r = (size_t)(sq.row0 + t0 + t);
      const float w = q == tid ? pw : a.o_norm[i], z = q == tid ? pz : silu(zs[t][c]);
      const float o = __fmul_rn(__fmul_rn(__fmul_rn(OUT[t][i], inv_o[t]), w), z);
      a.oq[r * a.vdim + h * VD + i] = warp_quant32(o, &a.os[r * (a.vdim / 32) + (h * VD) / 32 + (i >> 5)]);
    }
    __syncthreads();
  }
  if (!a.adv) {
    const size_t off = seq_off + (size_t)sq.base_slot * a.slot_stride_q + head_off;
    if (tid < SQ) {
      const int row = tid / (VC / 16), c16 = tid - row * (VC / 16);
      const size_t o = off + (size_t)row * VD + vcol0 + c16 * 16;
      *reinterpret_cast<int4*>(a.st_hi + o) = *reinterpret_cast<const int4*>(&hi[row][c16 * 16]);
      *reinterpret_cast<int4*>(a.st_lo + o) = *reinterpret_cast<const int4*>(&lo[row][c16 * 16]);
    }
    if (tid < KD * GPC) a.st_sc[off / 32 + (tid / GPC) * (VD / 32) + grp * GPC + tid % GPC] = sc[tid / GPC][tid % GPC];
    if (tid < 3 * KD && grp == 0) {
      float* d = cst0 + (size_t)sq.base_slot * a.conv_slot_stride;
      d[0] = c0; d[1] = c1; d[2] = c2;
    }
  }
}

// One CTA per (head, sequence).
template <int NTH>
__global__ void __launch_bounds__(NTH, NTH == 256 ? 4 : 2) kda_recur_kernel(const KdaArgs a) {
  kda_layer<NTH, 1>(a);
}

// Two CTAs per (head, sequence), one per value group (grid x = 2 * heads).
template <int NTH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTH, 1) kda_recur_split_kernel(const KdaArgs a) {
  kda_layer<NTH, 2>(a);
}

// ---------------------------------------------------------------- MoE

// Router of one token row, run by one warp (src/ops_moe.c:12-163): sigmoid
// scores, key = score + bias, top-k by key (first index on ties), weights =
// the scores renormalised by their sequential sum in selection order.
// Every lane returns the experts (-1: none left) and weights in sel_e /
// sel_w[0..topk).  E <= 256, topk <= 16.
LZ_HD void route_row(const float* __restrict__ logits, const float* __restrict__ bias, int E, int topk,
                     int* sel_e, float* sel_w) {
  const int lane = threadIdx.x & 31;
  float score[8], key[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = lane + 32 * j;
    if (e < E) {
      score[j] = sigmoid(logits[e]);
      key[j] = __fadd_rn(score[j], bias[e]);
    } else {
      score[j] = 0.0f;
      key[j] = -1e30f;
    }
  }
  float wsum = 0.0f;
  for (int t = 0; t < topk; t++) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int e = lane + 32 * j;
      if (e < E && key[j] > -1e30f) {
        const unsigned long long kk = ((unsigned long long)fkey(key[j]) << 32) | (0xFFFFFFFFu - (uint32_t)e);
        best = kk > best ? kk : best;
      }
    }
    best = warp_max_u64(best);
    const int bi = best ? argmax_index(best) : -1;
    float sw = 0.0f;
    if (bi >= 0 && (bi & 31) == lane) {
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j == (bi >> 5)) { sw = score[j]; key[j] = -1e30f; }
    }
    sw = __shfl_sync(0xffffffffu, sw, bi >= 0 ? (bi & 31) : 0);
    wsum = __fadd_rn(wsum, bi >= 0 ? sw : 0.0f);
    sel_e[t] = bi;
    sel_w[t] = bi >= 0 ? sw : 0.0f;
  }
  for (int t = 0; t < topk; t++)
    if (wsum > 0.0f && sel_e[t] >= 0) sel_w[t] = __fdiv_rn(sel_w[t], wsum);
}

// Router of one token row (route_row, warp 0) into pair_expert / pair_w;
// then the per-32 quantisation of the row's latent (src/forward_moe.c:150)
// and of the shared expert's silu(gate) * up (src/forward_moe.c:484-536)
// by all warps.  The path for more than 8 token rows.
__global__ void moe_route_kernel(const float* __restrict__ moein, int ldm, int off_router, int off_lat,
                                 const float* __restrict__ bias, int E, int topk, int latent,
                                 int* pair_expert, float* pair_w, int8_t* latq, float* lats,
                                 int off_shg, int off_shu, int sw, int8_t* shq, float* shs) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) {
    int se[16];
    float sw_[16];
    route_row(moein + (size_t)r * ldm + off_router, bias, E, topk, se, sw_);
    if (lane < topk) {
      for (int t = 0; t < 16; t++)
        if (t == lane) {
          pair_expert[r * topk + t] = se[t];
          pair_w[r * topk + t] = sw_[t];
        }
    }
  }
  const int ng_l = latent / 32, ng_s = sw / 32;
  for (int g = warp; g < ng_l + ng_s; g += blockDim.x >> 5) {
    if (g < ng_l) {
      const float v = moein[(size_t)r * ldm + off_lat + g * 32 + lane];
      latq[(size_t)r * latent + g * 32 + lane] = warp_quant32(v, &lats[(size_t)r * ng_l + g]);
    } else {
      const int gg = g - ng_l, i = gg * 32 + lane;
      const float gv = moein[(size_t)r * ldm + off_shg + i], uv = moein[(size_t)r * ldm + off_shu + i];
      shq[(size_t)r * sw + i] = warp_quant32(__fmul_rn(silu(gv), uv), &shs[(size_t)r * ng_s + gg]);
    }
  }
}

// Router and w1/w3 of one (token, expert) pair in one kernel, for at most
// 8 token rows (the pair's expert is known only after the routing, so a
// separate router launch sat on the critical path of every layer).  Block
// (chunk, pair p): warp 0 routes the pair's row (route_row) while the other
// warps quantise the row's latent per 32 into shared memory; blocks of
// chunk 0 store the row's experts and weights for w2 and the combine;
// blocks of the row's first pair quantise their share of the shared
// expert's silu(gate) * up.  Then FC = 64 * 16 / LPR consecutive FFN
// outputs of w1 and of w3: int8 GEMV over the latent with LPR lanes per
// weight row (LPR = 16 for latent <= 512: two rows per warp at a time),
// silu(w1.x) * (w3.x), the per-32 quantisation of each group
// (src/forward_moe.c:189-196).  w13 is the expert's [w1 rows; w3 rows]
// ([2 ffn][latent]); latent <= 32 * LPR.
template <int LPR>
__global__ void __launch_bounds__(256)
moe_route_w13_kernel(const float* __restrict__ moein, int ldm, int off_router, int off_lat,
                     const float* __restrict__ bias, int E, int topk,
                     const int8_t* __restrict__ w13q, const float* __restrict__ w13s, int ffn, int latent, int gs,
                     int* pair_expert, float* pair_w, int8_t* hq, float* hs,
                     int off_shg, int off_shu, int sw, int8_t* shq, float* shs) {
  constexpr int RPI = 32 / LPR;             // weight rows per warp per step
  constexpr int RW = 8 * RPI;               // weight rows per warp
  constexpr int FC = 8 * RW / 2;            // FFN outputs per block
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float P[8][RW][LPR];
  __shared__ float H[2 * FC];
  __shared__ __align__(16) int8_t lq[1024];
  __shared__ float ls[32];
  __shared__ int s_e[16];
  __shared__ float s_w[16];
  const int p = blockIdx.y, r = p / topk, t = p - r * topk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* row = moein + (size_t)r * ldm;
  const int nsb = latent / 32;
  if (warp == 0) {
    int se[16];
    float sw_[16];
    route_row(row + off_router, bias, E, topk, se, sw_);
    if (lane == 0)
      for (int i = 0; i < topk; i++) {
        s_e[i] = se[i];
        s_w[i] = sw_[i];
      }
  } else {
    for (int g = warp - 1; g < nsb; g += 7) lq[g * 32 + lane] = warp_quant32(row[off_lat + g * 32 + lane], &ls[g]);
  }
  if (t == 0 && sw) {
    // this block's share of the row's shared-expert groups (warp 0, the
    // router, takes them last)
    const int ng_s = sw / 32, per = (ng_s + gridDim.x - 1) / gridDim.x;
    for (int gg = blockIdx.x * per + (7 - warp); gg < min(ng_s, (blockIdx.x + 1) * per); gg += 8) {
      const int i = gg * 32 + lane;
      shq[(size_t)r * sw + i] = warp_quant32(__fmul_rn(silu(row[off_shg + i]), row[off_shu + i]),
                                             &shs[(size_t)r * ng_s + gg]);
    }
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x < topk && t == 0) {
    pair_expert[r * topk + threadIdx.x] = s_e[threadIdx.x];
    pair_w[r * topk + threadIdx.x] = s_w[threadIdx.x];
  }
  const int e = s_e[t];
  if (e < 0) return;
  const int rb = gs / 32, ng = latent / gs;
  const size_t wbase = (size_t)e * 2 * ffn * latent;
  const size_t sbase = (size_t)e * 2 * ffn * ng;
  const int sb = lane % LPR, half = lane / LPR;
  // local weight row lr < FC: w1 row chunk*FC + lr; else w3 row ffn + chunk*FC + lr - FC
  auto orow_of = [&](int lr) { return lr < FC ? blockIdx.x * FC + lr : ffn + blockIdx.x * FC + (lr - FC); };
  int4 xa = make_int4(0, 0, 0, 0), xb = xa;
  float xsv = 0.0f;
  if (sb < nsb) {
    xa = *reinterpret_cast<const int4*>(lq + sb * 32);
    xb = *reinterpret_cast<const int4*>(lq + sb * 32 + 16);
    xsv = ls[sb];
  }
  int4 wa[8], wb[8];
  float wsv[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const int orow = orow_of(warp * RW + k * RPI + half);
    if (sb < nsb) {
      const int8_t* wr = w13q + wbase + (size_t)orow * latent;
      wa[k] = __ldg(reinterpret_cast<const int4*>(wr + sb * 32));
      wb[k] = __ldg(reinterpret_cast<const int4*>(wr + sb * 32 + 16));
      wsv[k] = rb == 1 ? __ldg(w13s + sbase + (size_t)orow * ng + sb) : 0.0f;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; k++)
    if (sb < nsb) {
      const float a = (float)dot32(wa[k], wb[k], xa, xb);
      P[warp][k * RPI + half][sb] = rb > 1 ? __fmul_rn(a, xsv) : __fmul_rn(a, __fmul_rn(xsv, wsv[k]));
    }
  __syncwarp();
  if (lane < RW) {
    const int lr = warp * RW + lane;
    H[lr] = q8_reduce(P[warp][lane], w13s + sbase + (size_t)orow_of(lr) * ng, rb, ng);
  }
  __syncthreads();
  if (warp < FC / 32) {
    const int j = warp * 32 + lane;
    const float a = __fmul_rn(silu(H[j]), H[FC + j]);
    hq[(size_t)p * ffn + blockIdx.x * FC + j] = warp_quant32(a, &hs[(size_t)p * (ffn / 32) + blockIdx.x * (FC / 32) + warp]);
  }
}

// Element i of a token row's latent output: the sum over its selected
// experts, in selection order, of w * (the pair's w2 row) (src/forward_moe.c:
// 198-199); unrouted pairs (expert -1) are skipped.  e / w are the row's
// experts and weights (shared memory); the pair rows are loaded four at a
// time ahead of their adds (the rows are in bounds whether routed or not).
// CG reads them through L2 only (rows written by other blocks of the same
// kernel).
template <bool CG>
LZ_HD float combine_elem(const int* e, const float* w, int topk, const float* __restrict__ h2, int latent, int i) {
  float acc = 0.0f;
  for (int t0 = 0; t0 < topk; t0 += 4) {
    float h[4];
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (t0 + u < topk) h[u] = CG ? __ldcg(h2 + (size_t)(t0 + u) * latent + i) : h2[(size_t)(t0 + u) * latent + i];
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (t0 + u < topk && e[t0 + u] >= 0) acc = __fadd_rn(acc, __fmul_rn(w[t0 + u], h[u]));
  }
  return acc;
}

// w2 (latent x ffn) of every pair, two output rows per warp (16 outputs
// per block, so batch 1 runs in one wave of blocks), ffn <= 2048; for each
// token row and 32-output group, the last of the blocks producing it (2
// per pair) forms that group of lat_y = sum over the row's selected
// experts, in selection order, of w * h2 (src/forward_moe.c:198-199) and
// quantises it per 32.
constexpr int kW2Rows = 2;   // output rows per warp
__global__ void __launch_bounds__(256)
moe_w2_kernel(const int8_t* __restrict__ w2q, const float* __restrict__ w2s, int ffn, int latent, int gs,
              const int* __restrict__ pair_expert, const float* __restrict__ pair_w, int topk,
              const int8_t* __restrict__ hq, const float* __restrict__ hs, float* h2,
              int* row_counter, int8_t* yq, float* ys) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float P[8][kW2Rows][64];
  __shared__ int s_last;
  const int p = blockIdx.y, r = p / topk;
  const int e = pair_expert[p];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * 8 + warp) * kW2Rows;
  if (e >= 0 && n0 < latent) {
    const int nsb = ffn / 32, rb = gs / 32, ng = ffn / gs;
    const int8_t* xr = hq + (size_t)p * ffn;
    const float* xsr = hs + (size_t)p * nsb;
    int4 wa[kW2Rows][2], wb[kW2Rows][2];
    float wsv[kW2Rows][2];
#pragma unroll
    for (int q = 0; q < kW2Rows; q++)
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const int s = lane + 32 * j, n = n0 + q;
        if (s < nsb && n < latent) {
          const int8_t* wr = w2q + ((size_t)e * latent + n) * ffn;
          wa[q][j] = __ldg(reinterpret_cast<const int4*>(wr + s * 32));
          wb[q][j] = __ldg(reinterpret_cast<const int4*>(wr + s * 32 + 16));
          wsv[q][j] = rb == 1 ? __ldg(w2s + ((size_t)e * latent + n) * ng + s) : 0.0f;
        }
      }
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int s = lane + 32 * j;
      if (s < nsb) {
        const int4 xa = __ldg(reinterpret_cast<const int4*>(xr + s * 32));
        const int4 xb = __ldg(reinterpret_cast<const int4*>(xr + s * 32 + 16));
        const float xsv = __ldg(xsr + s);
#pragma unroll
        for (int q = 0; q < kW2Rows; q++)
          if (n0 + q < latent) {
            const float a = (float)dot32(wa[q][j], wb[q][j], xa, xb);
            P[warp][q][s] = rb > 1 ? __fmul_rn(a, xsv) : __fmul_rn(a, __fmul_rn(xsv, wsv[q][j]));
          }
      }
    }
    __syncwarp();
    if (lane < kW2Rows && n0 + lane < latent) {
      const int n = n0 + lane;
      h2[(size_t)p * latent + n] = q8_reduce(P[warp][lane], w2s + ((size_t)e * latent + n) * ng, rb, ng);
    }
  }
  // the last of the blocks that produce 32-output group g of row r (2 per
  // pair) forms that group's combine (one warp)
  constexpr int BPG = 32 / (8 * kW2Rows);
  __threadfence();
  __syncthreads();
  const int g = blockIdx.x / BPG, cidx = r * (latent / 32) + g;
  if (threadIdx.x == 0) {
    const int nb = min(BPG, (int)gridDim.x - BPG * g);
    s_last = atomicAdd(row_counter + cidx, 1) == topk * nb - 1;
  }
  __syncthreads();
  if (!s_last || warp != 0) return;
  __threadfence();
  int pe = -1;
  float pw = 0.0f;
  if (lane < topk) {
    pe = __ldcg(pair_expert + r * topk + lane);
    pw = __ldcg(pair_w + r * topk + lane);
  }
  __shared__ int s_pe[16];
  __shared__ float s_pw[16];
  if (lane < topk) {
    s_pe[lane] = pe;
    s_pw[lane] = pw;
  }
  __syncwarp();
  const float acc = combine_elem<true>(s_pe, s_pw, topk, h2 + (size_t)r * topk * latent, latent, g * 32 + lane);
  yq[(size_t)r * latent + g * 32 + lane] = warp_quant32(acc, &ys[(size_t)r * (latent / 32) + g]);
  if (lane == 0) row_counter[cidx] = 0;
}

// ------------------------------------------------ grouped experts (R > 8)
//
// With many token rows the (token, expert) pairs are bucketed by expert
// into tiles of at most 16 pair rows; each tile runs the warp-tile
// tensor-core GEMM over its expert's weights, so every expert's weights
// are streamed once per 16 rows instead of once per pair.  The arithmetic
// per pair is that of moe_route_w13_kernel / moe_w2_kernel.

struct MoeTile {
  int e, start, count;
};

// Buckets the P pairs by expert: list holds pair indices grouped by
// expert, tiles the (expert, start, count) of every tile of at most trows
// pairs, *ntiles their number.  Pairs with a negative expert are skipped.
// One block; E <= 256, P <= 1024 kMoeGroupPer.
constexpr int kMoeGroupPer = 8;
__global__ void __launch_bounds__(1024) moe_group_kernel(const int* __restrict__ pair_expert, int P, int E,
                                                         int* list, MoeTile* tiles, int* ntiles, int trows) {
  pdl_trigger();
  pdl_wait();
  __shared__ int cnt[256], off[256];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  int slot[kMoeGroupPer], ex[kMoeGroupPer];
#pragma unroll
  for (int k = 0; k < kMoeGroupPer; k++) {
    const int p = threadIdx.x + k * blockDim.x;
    slot[k] = -1;
    ex[k] = -1;
    if (p < P) {
      ex[k] = pair_expert[p];
      if (ex[k] >= 0) slot[k] = atomicAdd(&cnt[ex[k]], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0, nt = 0;
    for (int e = 0; e < E; e++) {
      off[e] = o;
      for (int i = 0; i < cnt[e]; i += trows) tiles[nt++] = MoeTile{e, o + i, min(trows, cnt[e] - i)};
      o += cnt[e];
    }
    *ntiles = nt;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kMoeGroupPer; k++)
    if (slot[k] >= 0) list[off[ex[k]] + slot[k]] = threadIdx.x + k * blockDim.x;
}

// w1/w3 of one tile: each warp 32 FFN outputs (4 n tiles of w1 rows, 4 of
// w3 rows) for the tile's pair rows, then silu(w1.x) * (w3.x) quantised per
// 32 into hq / hs of each pair.  Grid (ffn / 128, max tiles), 128 threads.
template <bool RB1>
__global__ void __launch_bounds__(128)
moe_w13_group_kernel(const int8_t* __restrict__ w13q, const float* __restrict__ w13s, int ffn, int latent,
                     int gs, const int* __restrict__ list, const MoeTile* __restrict__ tiles,
                     const int* __restrict__ ntiles, int topk, const int8_t* __restrict__ latq,
                     const float* __restrict__ lats, int8_t* hq, float* hs) {
  pdl_trigger();
  pdl_wait();
  if ((int)blockIdx.y >= *ntiles) return;
  const MoeTile T = tiles[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int j0 = (blockIdx.x * 4 + warp) * 32;
  if (j0 >= ffn) return;
  const int ng = latent / gs;
  if (lane == 0) {   // the rest of the warp's w1 and w3 rows stream into L2 meanwhile
    const size_t eo = (size_t)T.e * 2 * ffn;
    const int rows = min(32, ffn - j0);
    prefetch_l2(w13q + (eo + j0) * latent, (size_t)rows * latent);
    prefetch_l2(w13q + (eo + ffn + j0) * latent, (size_t)rows * latent);
    prefetch_l2(w13s + (eo + j0) * ng, (size_t)rows * ng * 4);
    prefetch_l2(w13s + (eo + ffn + j0) * ng, (size_t)rows * ng * 4);
  }
  const int pa = list[T.start + min(gid, T.count - 1)], pc = list[T.start + min(gid + 8, T.count - 1)];
  int nb[8];
#pragma unroll
  for (int t = 0; t < 8; t++) nb[t] = t < 4 ? j0 + 8 * t : ffn + j0 + 8 * (t - 4);
  RedState<RB1> st[8][4];
  wmma_pass<8, RB1>(w13q + (size_t)T.e * 2 * ffn * latent, w13s + (size_t)T.e * 2 * ffn * ng, 2 * ffn, latent, gs,
                    latq, lats, pa / topk, pc / topk, nb, st);
  // rows g (e < 2) and g+8 (e >= 2): 8 values each per lane, 32 per row
  // across the 4 lanes of the row
#pragma unroll
  for (int half = 0; half < 2; half++) {
    float h[8];
    uint32_t am = 0;
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const int e = half * 2 + c;
        h[t * 2 + c] = __fmul_rn(silu(mma_result(st[t][e])), mma_result(st[t + 4][e]));
        const uint32_t b = abs_bits(h[t * 2 + c]);
        am = am > b ? am : b;
      }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      const uint32_t w = __shfl_xor_sync(0xffffffffu, am, o);
      am = am > w ? am : w;
    }
    float sg, inv;
    q8_scale_from_amax(am, &sg, &inv);
    const int row = gid + half * 8;
    if (row < T.count) {
      const int p = half ? pc : pa;
#pragma unroll
      for (int t = 0; t < 4; t++)
#pragma unroll
        for (int c = 0; c < 2; c++)
          hq[(size_t)p * ffn + j0 + t * 8 + tq * 2 + c] = (int8_t)q8_clamp(q8_round(__fmul_rn(h[t * 2 + c], inv)));
      if (tq == 0) hs[(size_t)p * (ffn / 32) + j0 / 32] = sg;
    }
  }
}

// w2 of one tile: each warp 16 latent outputs of the tile's pair rows into
// h2 (pair x latent).  Grid (latent / 64, max tiles), 128 threads.
template <bool RB1>
__global__ void __launch_bounds__(128)
moe_w2_group_kernel(const int8_t* __restrict__ w2q, const float* __restrict__ w2s, int ffn, int latent, int gs,
                    const int* __restrict__ list, const MoeTile* __restrict__ tiles,
                    const int* __restrict__ ntiles, const int8_t* __restrict__ hq, const float* __restrict__ hs,
                    float* h2) {
  pdl_trigger();
  pdl_wait();
  if ((int)blockIdx.y >= *ntiles) return;
  const MoeTile T = tiles[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int n0 = (blockIdx.x * 4 + warp) * 16;
  if (n0 >= latent) return;
  const int ng = ffn / gs;
  if (lane == 0) {
    const int rows = min(16, latent - n0);
    prefetch_l2(w2q + ((size_t)T.e * latent + n0) * ffn, (size_t)rows * ffn);
    prefetch_l2(w2s + ((size_t)T.e * latent + n0) * ng, (size_t)rows * ng * 4);
  }
  const int pa = list[T.start + min(gid, T.count - 1)], pc = list[T.start + min(gid + 8, T.count - 1)];
  int nb[2] = {n0, n0 + 8};
  RedState<RB1> st[2][4];
  wmma_pass<2, RB1>(w2q + (size_t)T.e * latent * ffn, w2s + (size_t)T.e * latent * ng, latent, ffn, gs, hq, hs, pa,
                    pc, nb, st);
#pragma unroll
  for (int t = 0; t < 2; t++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int row = gid + (e >= 2 ? 8 : 0);
      const int o = n0 + t * 8 + tq * 2 + (e & 1);
      if (row < T.count && o < latent) h2[(size_t)(e >= 2 ? pc : pa) * latent + o] = mma_result(st[t][e]);
    }
}

// ------------------------------------- TMA-staged grouped expert kernels
//
// The grouped w1/w3 and w2 products with the roles of the MMA operands
// swapped: the expert's weight rows are the 16-row A operand, streamed by
// 2-D TMA loads (128-byte K slices, 128-byte swizzle) through an mbarrier
// ring, and the tile's <= 8 gathered activation rows (token rows of latq
// for w1/w3, pair rows of hq for w2) are the 8-column B operand, copied
// once into a resident swizzled buffer.  With about 8 pairs per expert this
// wastes no MMA rows on padding.  Each (output, pair) keeps the reference
// float epilogue in K order.  Block = CW consumer warps of MW 16-row weight
// tiles each + one producer warp; grid (output chunks of 128, tiles).
constexpr int kMoeTileRows = 8;   // pairs per tile on this path

struct alignas(64) MoeTmaArgs {
  CUtensorMap wq;            // stacked expert weights [E * rows_e][K] u8
  CUtensorMap wsc;           // their scales [E * rows_e][K/32] f32 (gs = 32 only)
  const float* ws;           // scales read directly (gs > 32)
  const int* list;
  const MoeTile* tiles;
  const int* ntiles;
  const int8_t* xq;          // activation rows: latq (w1/w3) or hq (w2)
  const float* xs;
  int8_t* hq;                // w1/w3 outputs: silu(w1 x) * (w3 x) quantised per 32
  float* hs;
  float* h2;                 // w2 outputs [pair][latent]
  int* err;
  int K, gs, rows_e, ffn, latent, topk;
};

template <bool W13, bool RB1>
struct MoeTma {
  static constexpr int CW = 4;                      // consumer warps
  static constexpr int MW = W13 ? 4 : 2;            // 16-row weight tiles per warp (w13: 2 of w1 + 2 of w3)
  static constexpr int BOX = 128;                   // weight rows per box (w13: a w1 box and a w3 box)
  static constexpr int NBOX = W13 ? 2 : 1;
  static constexpr int NST = W13 ? 2 : 3;          // w13: two stages let 3 blocks fit per SM (measured faster)
  static constexpr int B = NBOX * BOX * 128;        // swizzled weight tile per stage
  static constexpr int WS = RB1 ? NBOX * BOX * 16 : 0;
  static constexpr int KMAX = 2048;
  // bytes of dynamic shared memory for inner dimension K
  static size_t smem(int K) { return 1024 + (size_t)NST * (B + WS) + 8 * (size_t)K + 8 * (K / 32) * 4 + 2 * NST * 8; }
};

template <bool W13, bool RB1, int GM>
__global__ void __launch_bounds__((MoeTma<W13, RB1>::CW + 1) * 32) moe_tma_kernel(const __grid_constant__ MoeTmaArgs p) {
  using C = MoeTma<W13, RB1>;
  constexpr int CW = C::CW, MW = C::MW, NST = C::NST;
  extern __shared__ uint8_t moe_smem[];
  const int K = p.K, nsb = K >> 5, nit = K >> 7;
  const uint32_t raw = smem_u32(moe_smem);
  const uint32_t base = (raw + 1023u) & ~1023u;       // NST weight tiles
  const uint32_t wsb = base + NST * C::B;             // weight-scale boxes (gs = 32)
  const uint32_t bbase = wsb + NST * C::WS;           // resident B: K/128 slices of 8 rows x 128 B
  const uint32_t xsb = bbase + 8 * K;                 // activation scales [8][K/32]
  const uint32_t bars = xsb + 8 * nsb * 4;
  uint8_t* gen = moe_smem + (base - raw);
  pdl_trigger();
  pdl_wait();
  if ((int)blockIdx.y >= *p.ntiles) return;
  const MoeTile T = p.tiles[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = blockIdx.x * 128;      // first j (w1/w3) or latent output (w2) of the block
  const int erow = T.e * p.rows_e;
  if (threadIdx.x == CW * 32) {
    for (int s = 0; s < NST; s++) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (NST + s), CW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](int it) {
    const int stg = it % NST;
    const uint32_t full = bars + 8 * stg, tile = base + stg * C::B;
    mbar_expect_tx(full, C::B + C::WS);
#pragma unroll
    for (int b = 0; b < C::NBOX; b++) {
      const int row = erow + o0 + b * p.ffn;
      tma_load_2d(tile + b * C::BOX * 128, &p.wq, it * 128, row, full);
      if (RB1) tma_load_2d(wsb + stg * C::WS + b * C::BOX * 16, &p.wsc, it * 4, row, full);
    }
  };
  if (threadIdx.x == CW * 32)
    for (int it = g_dbg_skip_stage ? 1 : 0; it < min(nit, NST); it++) issue(it);   // the hook skips stage 0
  // resident activation rows of the tile (rows past the count repeat the last)
  {
    const int cpr = K >> 4;   // 16-byte chunks per row
    for (int idx = threadIdx.x; idx < 8 * cpr; idx += blockDim.x) {
      const int r = idx / cpr, j = idx - r * cpr;
      const int pr = p.list[T.start + min(r, T.count - 1)];
      const int src = W13 ? pr / p.topk : pr;
      const uint4 v = *reinterpret_cast<const uint4*>(p.xq + (size_t)src * K + j * 16);
      *reinterpret_cast<uint4*>(gen + (bbase - base) + (j >> 3) * 1024 + r * 128 + (((j & 7) ^ r) << 4)) = v;
    }
    float* xsm = reinterpret_cast<float*>(gen + (xsb - base));
    for (int idx = threadIdx.x; idx < 8 * nsb; idx += blockDim.x) {
      const int r = idx / nsb, c = idx - r * nsb;
      const int pr = p.list[T.start + min(r, T.count - 1)];
      const int src = W13 ? pr / p.topk : pr;
      xsm[idx] = p.xs[(size_t)src * nsb + c];
    }
  }
  __syncthreads();
  if (warp == CW) {
    if (lane != 0) return;
    bool ok = true;
    int it = min(nit, NST);
    for (; it < nit; it++) {
      if (!mbar_wait(bars + 8 * (NST + it % NST), (it / NST - 1) & 1)) {
        ok = false;
        break;
      }
      fence_proxy_async_smem();
      issue(it);
    }
    if (!ok) atomicExch(p.err, 1);
    for (int j = max(0, it - NST); j < it; j++) mbar_wait(bars + 8 * (j % NST), (j / NST) & 1);
    return;
  }
  const int gid = lane >> 2, tq = lane & 3, sw = lane & 7;
  // stage row of weight tile i of this warp: w13 tiles 0, 1 in the w1 box,
  // 2, 3 the same j in the w3 box; w2 tiles i
  auto trow = [&](int i) { return W13 ? (i >> 1) * C::BOX + warp * 32 + (i & 1) * 16 : warp * 32 + i * 16; };
  const int rb = p.gs >> 5, ng = K / p.gs;
  int grow[MW][2];   // stacked-tensor weight rows of fragment rows gid, gid + 8
  float wrow[MW][2];
#pragma unroll
  for (int i = 0; i < MW; i++)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int r = trow(i) + gid + 8 * h;
      const int b = W13 ? r / C::BOX : 0;
      grow[i][h] = erow + o0 + b * p.ffn + (r - b * C::BOX);
      wrow[i][h] = GM == 1 ? __ldg(p.ws + grow[i][h]) : 0.0f;
    }
  RedState<RB1> st[MW][4];
#pragma unroll
  for (int i = 0; i < MW; i++)
#pragma unroll
    for (int e = 0; e < 4; e++)
#pragma unroll
      for (int j = 0; j < (RB1 ? 4 : 2); j++) st[i][e].a[j] = 0.0f;
  uint32_t aoff[MW];
#pragma unroll
  for (int i = 0; i < MW; i++) aoff[i] = (uint32_t)(trow(i) + sw + (((lane >> 3) & 1) << 3)) * 128u;
  const int ach = lane >> 4, bch = (lane >> 3) & 1;
  const uint32_t boff = (uint32_t)sw * 128u;
  const float* xsm = reinterpret_cast<const float*>(gen + (xsb - base));
  int gcnt = 0, gidx = 0;
  bool ok = true;
#pragma unroll 1
  for (int it = 0; it < nit; it++) {
    const int stg = it % NST;
    if (!mbar_wait(bars + 8 * stg, (it / NST) & 1)) {
      ok = false;
      break;
    }
    const uint32_t tile = base + stg * C::B, bslice = bbase + it * 1024;
    const float* wsm = reinterpret_cast<const float*>(gen + (wsb - base) + stg * C::WS);
    unsigned af[4][MW][4], bf[4][2];
#pragma unroll
    for (int sl = 0; sl < 4; sl++) {
      ldsm_x2(bslice + boff + ((uint32_t)((2 * sl + bch) ^ sw) << 4), bf[sl][0], bf[sl][1]);
#pragma unroll
      for (int i = 0; i < MW; i++)
        ldsm_x4(tile + aoff[i] + ((uint32_t)((2 * sl + ach) ^ sw) << 4), af[sl][i][0], af[sl][i][1], af[sl][i][2],
                af[sl][i][3]);
    }
    float4 wv[MW][2];
    if (RB1) {
#pragma unroll
      for (int i = 0; i < MW; i++)
#pragma unroll
        for (int h = 0; h < 2; h++) wv[i][h] = *reinterpret_cast<const float4*>(wsm + (trow(i) + gid + 8 * h) * 4);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bars + 8 * (NST + stg));   // the stage is in registers
#pragma unroll
    for (int sl = 0; sl < 4; sl++) {
      const int s = it * 4 + sl;
      const float x0 = xsm[(2 * tq) * nsb + s], x1 = xsm[(2 * tq + 1) * nsb + s];
      bool gend = false;
      float wg[MW][2];
      if (GM == 1) {
        gend = s == nsb - 1;
#pragma unroll
        for (int i = 0; i < MW; i++) wg[i][0] = wrow[i][0], wg[i][1] = wrow[i][1];
      } else if (GM == 2) {
        gend = ++gcnt == rb;
        if (gend) {
          gcnt = 0;
#pragma unroll
          for (int i = 0; i < MW; i++)
#pragma unroll
            for (int h = 0; h < 2; h++) wg[i][h] = __ldg(p.ws + (size_t)grow[i][h] * ng + gidx);
          gidx++;
        }
      } else {
#pragma unroll
        for (int i = 0; i < MW; i++)
#pragma unroll
          for (int h = 0; h < 2; h++) wg[i][h] = f4_at(wv[i][h], sl);
      }
#pragma unroll
      for (int i = 0; i < MW; i++) {
        int d[4];
        mma_s8(d, af[sl][i], bf[sl][0], bf[sl][1]);
        // d[e]: weight row gid + 8 (e >> 1), pair column 2 tq + (e & 1)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float a = i2f_small(d[e]);
          const float xsv = (e & 1) ? x1 : x0;
          RedState<RB1>& R_ = st[i][e];
          if (!RB1) {
            R_.a[0] = __fadd_rn(R_.a[0], __fmul_rn(a, xsv));
            if (gend) {
              R_.a[1] = __fadd_rn(R_.a[1], __fmul_rn(R_.a[0], wg[i][e >> 1]));
              R_.a[0] = 0.0f;
            }
          } else {
            R_.a[sl] = __fadd_rn(R_.a[sl], __fmul_rn(a, __fmul_rn(xsv, wg[i][e >> 1])));
          }
        }
      }
    }
  }
  if (!ok) {
    atomicExch(p.err, 1);
    return;
  }
  int pr[2];
#pragma unroll
  for (int c = 0; c < 2; c++) pr[c] = p.list[T.start + min(2 * tq + c, T.count - 1)];
  if (W13) {
    // per pair column c: the warp's 32 j values sit in the 8 lanes of equal
    // tq (tiles i = 0, 1; rows gid and gid + 8): silu(w1) * w3, amax over
    // those lanes, per-32 quantisation (src/forward_moe.c:434-545)
    const int j0 = o0 + warp * 32;
#pragma unroll
    for (int c = 0; c < 2; c++) {
      float h[4];
      uint32_t am = 0;
#pragma unroll
      for (int i = 0; i < 2; i++)
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          const int e = hh * 2 + c;
          h[i * 2 + hh] = __fmul_rn(silu(mma_result(st[i][e])), mma_result(st[i + 2][e]));
          const uint32_t b = abs_bits(h[i * 2 + hh]);
          am = am > b ? am : b;
        }
#pragma unroll
      for (int o = 4; o <= 16; o <<= 1) {
        const uint32_t w = __shfl_xor_sync(0xffffffffu, am, o);
        am = am > w ? am : w;
      }
      float sg, inv;
      q8_scale_from_amax(am, &sg, &inv);
      if (2 * tq + c < T.count) {
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
          for (int hh = 0; hh < 2; hh++)
            p.hq[(size_t)pr[c] * p.ffn + j0 + i * 16 + hh * 8 + gid] =
                (int8_t)q8_clamp(q8_round(__fmul_rn(h[i * 2 + hh], inv)));
        if (gid == 0) p.hs[(size_t)pr[c] * (p.ffn / 32) + j0 / 32] = sg;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < MW; i++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int c = e & 1;
        const int o = o0 + warp * 32 + i * 16 + gid + 8 * (e >> 1);
        if (2 * tq + c < T.count && o < p.latent) p.h2[(size_t)pr[c] * p.latent + o] = mma_result(st[i][e]);
      }
  }
}

// lat_y of one token row = sum over its selected experts, in selection
// order, of w * h2 (src/forward_moe.c:198-199), quantised per 32.
__global__ void moe_combine_kernel(const int* __restrict__ pair_expert, const float* __restrict__ pair_w, int topk,
                                   const float* __restrict__ h2, int latent, int8_t* yq, float* ys) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_pe[16];
  __shared__ float s_pw[16];
  if (threadIdx.x < topk) {
    s_pe[threadIdx.x] = pair_expert[r * topk + threadIdx.x];
    s_pw[threadIdx.x] = pair_w[r * topk + threadIdx.x];
  }
  __syncthreads();
  for (int g = warp; g < latent / 32; g += blockDim.x >> 5) {
    const float acc = combine_elem<false>(s_pe, s_pw, topk, h2 + (size_t)r * topk * latent, latent, g * 32 + lane);
    yq[(size_t)r * latent + g * 32 + lane] = warp_quant32(acc, &ys[(size_t)r * (latent / 32) + g]);
  }
}

// ---------------------------------------------------------------- MTP

// fc input of the draft head for one row: [rmsnorm_e(embed(tok)) |
// rmsnorm_h(hidden)] quantised per 32 (src/forward_mtp.c:53-67, 580-597).
__global__ void mtp_front_kernel(const int8_t* __restrict__ eq, const float* __restrict__ es, int egs,
                                 int d, const int* __restrict__ tok,
                                 const float* __restrict__ hid, const int* __restrict__ hid_idx,
                                 const float* __restrict__ w_e, const float* __restrict__ w_h, float eps,
                                 int8_t* xq, float* xs) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float sm[];           // [2][d] rows, [2][d + 16] squares
  __shared__ float s_inv[2];
  const int r = blockIdx.x;
  const int hr = hid_idx ? hid_idx[r] : r;
  const size_t base = (size_t)tok[r] * d;
  // each thread's loads issued together, then its stores
  for (int i0 = threadIdx.x; i0 < d; i0 += kRowLoadU * blockDim.x) {
    int8_t qv[kRowLoadU];
    float sv[kRowLoadU], hv[kRowLoadU];
#pragma unroll
    for (int u = 0; u < kRowLoadU; u++) {
      const int i = i0 + u * blockDim.x;
      qv[u] = i < d ? eq[base + i] : (int8_t)0;
      sv[u] = i < d ? es[(base + i) / egs] : 0.0f;
      hv[u] = i < d ? hid[(size_t)hr * d + i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kRowLoadU; u++) {
      const int i = i0 + u * blockDim.x;
      if (i < d) {
        sm[i] = __fmul_rn((float)qv[u], sv[u]);
        sm[d + i] = hv[u];
      }
    }
  }
  __syncthreads();
  if (blockDim.x == 2 * kSplitGroup && d % 512 == 0) {
    // one 128-thread group per half (chain warps 0-1 and 6-7), squares
    // into sm[2d..4d+32)
    __shared__ SplitSumShared split[2];
    const int g = threadIdx.x / kSplitGroup, u = threadIdx.x - g * kSplitGroup;
    const float ss = seq_sumsq_split(sm + (size_t)g * d, sm + 2 * (size_t)d + (size_t)g * (d + 16), d, u, 2 * g, g, split[g]);
    if (u == 64 * g) s_inv[g] = rsqrt_body(__fadd_rn(__fdiv_rn(ss, (float)d), eps));
  } else {
    if (threadIdx.x == 0) s_inv[0] = rsqrt_body(__fadd_rn(__fdiv_rn(seq_sumsq(sm, d), (float)d), eps));
    if (threadIdx.x == 32) s_inv[1] = rsqrt_body(__fadd_rn(__fdiv_rn(seq_sumsq(sm + d, d), (float)d), eps));
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  // a warp's groups are independent: four in flight
#pragma unroll 4
  for (int g = warp; g < 2 * d / 32; g += nw) {
    const int i = g * 32 + lane;
    const int half = i >= d;
    const int ii = half ? i - d : i;
    const float wv = half ? w_h[ii] : w_e[ii];
    const float o = __fmul_rn(__fmul_rn(sm[i], s_inv[half]), __fadd_rn(1.0f, wv));
    xq[(size_t)r * 2 * d + i] = warp_quant32(o, &xs[(size_t)r * (2 * d / 32) + g]);
  }
}

// Per-head RMSNorm (1+w) then RoPE of the first rot dims, in place on a
// 64-wide shared vector; called by every thread of the block.
LZ_HD void head_norm_rope(float* v, const float* w, float eps, int hd, int rot,
                          const float* cs_row, float* s_inv) {
  const int i = threadIdx.x;
  if (i == 0) *s_inv = rsqrt_body(__fadd_rn(__fdiv_rn(seq_sumsq(v, hd), (float)hd), eps));
  __syncthreads();
  float o = 0.0f;
  if (i < hd) o = __fmul_rn(__fmul_rn(v[i], *s_inv), __fadd_rn(1.0f, w[i]));
  __syncthreads();
  if (i < hd) v[i] = o;
  __syncthreads();
  const int half = rot / 2;
  float nv = 0.0f;
  if (i < half) {
    const float c = cs_row[2 * i], sn = cs_row[2 * i + 1];
    nv = __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(v[i + half], sn));
  } else if (i < rot) {
    const int j = i - half;
    const float c = cs_row[2 * j], sn = cs_row[2 * j + 1];
    nv = __fadd_rn(__fmul_rn(v[i], c), __fmul_rn(v[j], sn));
  }
  __syncthreads();
  if (i < rot) v[i] = nv;
  __syncthreads();
}

struct MtpRow {            // one draft / prefill row of the MTP block
  int seq, pos, active;
};

// K/V side of the MTP attention for one (row, kv head): k RMSNorm, RoPE,
// Q8 write of k and v into the row's sequence cache at `pos`
// (src/forward_attn.c:909-965).  64 threads (hd = 64).
__global__ void mtp_kv_write_kernel(const float* __restrict__ qkv, int ldq, int off_k, int off_v,
                                    const MtpRow* __restrict__ rows, const float* __restrict__ k_norm,
                                    float eps, int hd, int rot, int kvd, const float* __restrict__ rope_cs,
                                    int8_t* kq, float* ks, int8_t* vq, float* vs,
                                    size_t cache_seq_stride) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float v[64];
  __shared__ float s_inv;
  const int h = blockIdx.x, r = blockIdx.y;
  const MtpRow row = rows[r];
  if (!row.active) return;
  const int i = threadIdx.x;
  v[i] = qkv[(size_t)r * ldq + off_k + h * hd + i];
  __syncthreads();
  head_norm_rope(v, k_norm, eps, hd, rot, rope_cs + (size_t)row.pos * rot, &s_inv);
  const size_t cb = (size_t)row.seq * cache_seq_stride + (size_t)row.pos * kvd;
  kq[cb + h * hd + i] = warp_quant32(v[i], &ks[cb / 32 + (h * hd) / 32 + (i >> 5)]);
  const float vv = qkv[(size_t)r * ldq + off_v + h * hd + i];
  vq[cb + h * hd + i] = warp_quant32(vv, &vs[cb / 32 + (h * hd) / 32 + (i >> 5)]);
}

// Gated attention of one (row, head) over the row's MTP cache t <= pos:
// q RMSNorm + RoPE, Q8 scores (32-element partial sums, sequential), the
// reference softmax (sequential sum), weighted V sum (sequential over t,
// V staged through shared memory in chunks), times sigmoid(gate), then
// per-32 quantisation for o_proj.  hd = 64.
// src/forward_attn.c:17-41, 206-640, src/ops_norm.c:903-985.
constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 256;
__global__ void __launch_bounds__(kAttnThreads)
mtp_attn_kernel(const float* __restrict__ qkv, int ldq, int qd,
                const MtpRow* __restrict__ rows, const float* __restrict__ q_norm,
                float eps, int hd, int rot, int kvd, int kv_mul,
                const float* __restrict__ rope_cs, float scale,
                const int8_t* __restrict__ kq, const float* __restrict__ ks,
                const int8_t* __restrict__ vq, const float* __restrict__ vs,
                size_t cache_seq_stride, int8_t* aq, float* as) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float att[];
  __shared__ __align__(16) float qh[64];
  __shared__ __align__(16) int8_t vch[kAttnChunk][64];
  __shared__ __align__(16) float vsc[kAttnChunk][2];
  __shared__ float s_red[2];
  __shared__ uint32_t wk[kAttnThreads / 32];
  const int h = blockIdx.x, r = blockIdx.y;
  const MtpRow row = rows[r];
  if (!row.active) return;
  const int i = threadIdx.x;
  const int kvh = h / kv_mul;
  const int pos = row.pos;
  if (i < hd) qh[i] = qkv[(size_t)r * ldq + (size_t)h * 2 * hd + i];
  __syncthreads();
  head_norm_rope(qh, q_norm, eps, hd, rot, rope_cs + (size_t)pos * rot, &s_red[0]);
  const size_t cb = (size_t)row.seq * cache_seq_stride;
  // the query in registers; two positions per step, their K rows loaded
  // together and their score chains interleaved (each in the reference's
  // order)
  float qr[64];
#pragma unroll
  for (int e = 0; e < 64; e++) qr[e] = qh[e];
  uint32_t bk = 0;
  for (int t = i; t <= pos; t += 2 * blockDim.x) {
    const int tb = t + blockDim.x;
    const bool two = tb <= pos;
    int4 k4[2][4];
    float sc2[2][2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int tu = u ? (two ? tb : t) : t;
      const int8_t* kt = kq + cb + (size_t)tu * kvd + kvh * hd;
      const float* kts = ks + (cb + (size_t)tu * kvd + kvh * hd) / 32;
#pragma unroll
      for (int c = 0; c < 4; c++) k4[u][c] = __ldg(reinterpret_cast<const int4*>(kt) + c);
      sc2[u][0] = __ldg(kts);
      sc2[u][1] = __ldg(kts + 1);
    }
    float sum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int dd = 0; dd < 64; dd += 32) {
      float acc[2] = {0.0f, 0.0f};
#pragma unroll
      for (int e = 0; e < 32; e++)
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const int8_t kv = reinterpret_cast<const int8_t*>(k4[u])[dd + e];
          acc[u] = __fadd_rn(acc[u], __fmul_rn(qr[dd + e], (float)kv));
        }
#pragma unroll
      for (int u = 0; u < 2; u++) sum[u] = __fadd_rn(sum[u], __fmul_rn(acc[u], sc2[u][dd ? 1 : 0]));
    }
#pragma unroll
    for (int u = 0; u < 2; u++) {
      if (u == 1 && !two) break;
      const float a = __fmul_rn(sum[u], scale);
      att[u ? tb : t] = a;
      const uint32_t k = fkey(a);
      bk = k > bk ? k : bk;
    }
  }
  bk = warp_max_u32(bk);
  if ((i & 31) == 0) wk[i >> 5] = bk;
  __syncthreads();
  if (i == 0) {
    uint32_t m = 0;
    for (int w = 0; w < kAttnThreads / 32; w++) m = wk[w] > m ? wk[w] : m;
    const uint32_t u = (m & 0x80000000u) ? (m & 0x7FFFFFFFu) : ~m;
    s_red[1] = __uint_as_float(u);
  }
  __syncthreads();
  const float mx = s_red[1];
  for (int t = i; t <= pos; t += blockDim.x) att[t] = exp_body(__fsub_rn(att[t], mx));
  __syncthreads();
  if (i == 0) {
    const float sum = seq_sum(att, pos + 1);
    s_red[0] = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
  }
  __syncthreads();
  const float inv = s_red[0];
  for (int t = i; t <= pos; t += blockDim.x) att[t] = __fmul_rn(att[t], inv);
  float out = 0.0f;
  for (int t0 = 0; t0 <= pos; t0 += kAttnChunk) {
    const int nt = min(kAttnChunk, pos + 1 - t0);
    __syncthreads();
    {
      // the chunk's V rows and scales: every load in flight before the
      // first store
      constexpr int LV = kAttnChunk * 4 / kAttnThreads, LS = kAttnChunk * 2 / kAttnThreads;
      int4 v4[LV];
      float s4[LS];
#pragma unroll
      for (int u = 0; u < LV; u++) {
        const int q = i + u * kAttnThreads, tt = q >> 2, c = q & 3;
        if (tt < nt) v4[u] = __ldg(reinterpret_cast<const int4*>(vq + cb + (size_t)(t0 + tt) * kvd + kvh * hd) + c);
      }
#pragma unroll
      for (int u = 0; u < LS; u++) {
        const int q = i + u * kAttnThreads, tt = q >> 1, c = q & 1;
        if (tt < nt) s4[u] = __ldg(vs + (cb + (size_t)(t0 + tt) * kvd + kvh * hd) / 32 + c);
      }
#pragma unroll
      for (int u = 0; u < LV; u++) {
        const int q = i + u * kAttnThreads, tt = q >> 2, c = q & 3;
        if (tt < nt) reinterpret_cast<int4*>(&vch[tt][0])[c] = v4[u];
      }
#pragma unroll
      for (int u = 0; u < LS; u++) {
        const int q = i + u * kAttnThreads, tt = q >> 1, c = q & 1;
        if (tt < nt) vsc[tt][c] = s4[u];
      }
    }
    __syncthreads();
    if (i < hd) {
      const int g = i >> 5;
      int tt = 0;
      // 16 products formed ahead of their adds (the adds stay in order)
      for (; tt + 16 <= nt; tt += 16) {
        float pr[16];
#pragma unroll
        for (int j = 0; j < 16; j++)
          pr[j] = __fmul_rn(__fmul_rn(att[t0 + tt + j], (float)vch[tt + j][i]), vsc[tt + j][g]);
#pragma unroll
        for (int j = 0; j < 16; j++) out = __fadd_rn(out, pr[j]);
      }
      for (; tt < nt; tt++) out = __fadd_rn(out, __fmul_rn(__fmul_rn(att[t0 + tt], (float)vch[tt][i]), vsc[tt][g]));
    }
  }
  if (i < hd) {
    out = __fmul_rn(out, sigmoid(qkv[(size_t)r * ldq + (size_t)h * 2 * hd + hd + i]));
    aq[(size_t)r * qd + h * hd + i] = warp_quant32(out, &as[(size_t)r * (qd / 32) + (h * hd) / 32 + (i >> 5)]);
  }
}

// ------------------------------------------------------- spec rounds

// SeqRound.dbg: the rounds' test-only switches of lz_spec_round
// (src/generate.c:827-844, 976-982).
constexpr int kDbgBreakRollback = 1;   // a rejecting round leaves the ring where the verify left it
constexpr int kDbgSkipCatchup = 2;     // no MTP catch-up rows

struct SeqRound {          // per-sequence round bookkeeping on the device
  unsigned long long rng;   // sampler xorshift64* state (src/sampler.c:185-203)
  float temp, topp;         // sampler temperature and top-p
  int anchor, anchor_pos, mtp_pos, ssm_slot;
  int k, n_accept, n_emit, dbg;
  int draft[8], out[8];
  int rounds, emitted, accepted, drafted;   // running totals
};

// After the acceptance of a round (src/generate.c:798-991, 1234-1377):
// counters, the state ring pointed at the accepted slot
// ((base + n_accept + 1) % depth, src/forward_ckpt.c), the catch-up rows
// (MTP cache rows of accepted drafts 1..n_accept-1), the MTP position and
// the next anchor.
LZ_HD void round_bookkeeping(SeqRound& s, int b, int n_accept, int k, int kmax, int row0, int depth, int seq_len,
                             MtpRow* catch_rows, int* catch_tok, int* catch_hidx) {
  s.n_accept = n_accept;
  s.n_emit = n_accept + 1;
  s.rounds += 1;
  s.emitted += n_accept + 1;
  s.accepted += n_accept;
  s.drafted += k;
  // the ring rollback: the verify advanced the ring by k + 1 slots; a
  // round that rejected a draft points it at slot base + n_accept + 1
  // instead (the known-bad control leaves it at base + k + 1)
  const bool broken = (s.dbg & kDbgBreakRollback) && n_accept < k;
  s.ssm_slot = (s.ssm_slot + (broken ? k : n_accept) + 1) % depth;
  for (int j = 0; j < kmax - 1; j++) {
    MtpRow cr;
    cr.seq = b;
    cr.pos = s.mtp_pos + 1 + j;
    cr.active = j < n_accept - 1 && cr.pos < seq_len && !(s.dbg & kDbgSkipCatchup);
    catch_rows[b * (kmax - 1) + j] = cr;
    catch_tok[b * (kmax - 1) + j] = s.out[j < 8 ? j : 0];
    catch_hidx[b * (kmax - 1) + j] = row0 + j;
  }
  s.mtp_pos += n_accept;
  s.anchor = s.out[n_accept];
  s.anchor_pos = s.anchor_pos + 1 + n_accept;
}

// Greedy acceptance of one round (src/generate.c:232-243, 798-991): the
// verify arg-max of every row, accept the agreeing draft prefix, point
// the state ring at the accepted slot, reseed the draft chain from the
// verify hidden row n_accept, set up the catch-up rows and advance the
// MTP position.
// One sequence's acceptance, by every thread of the calling block.
LZ_HD void greedy_accept_seq(SeqRound* sr, int b, int kmax, const unsigned long long* vmax, const float* vhid, int d,
                             float* chain, int depth, int seq_len, MtpRow* catch_rows, int* catch_tok,
                             int* catch_hidx) {
  SeqRound& s = sr[b];
  const int row0 = b * (kmax + 1);
  __shared__ int n_acc_s;
  if (threadIdx.x == 0) {
    const int k = s.k;
    int n_accept = k;
    for (int i = 0; i < k; i++) {
      s.out[i] = argmax_index(__ldcg(vmax + row0 + i));
      if (s.draft[i] != s.out[i]) { n_accept = i; break; }
    }
    if (n_accept == k) s.out[k] = argmax_index(__ldcg(vmax + row0 + k));
    round_bookkeeping(s, b, n_accept, k, kmax, row0, depth, seq_len, catch_rows, catch_tok, catch_hidx);
    n_acc_s = n_accept;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    chain[(size_t)b * d + i] = __ldcg(vhid + (size_t)(row0 + n_acc_s) * d + i);
  __syncthreads();
}

LZ_HD void greedy_accept_all(const GemvFuse& f) {
  for (int b = 0; b < f.nseq; b++)
    greedy_accept_seq(f.sr, b, f.kmax, f.amax, f.vhid, f.d, f.chain, f.depth, f.seq_len, f.catch_rows, f.catch_tok,
                      f.catch_hidx);
}

__global__ void spec_accept_greedy_kernel(SeqRound* sr, int nseq, int kmax,
                                          const unsigned long long* __restrict__ vmax,
                                          const float* __restrict__ vhid, int d, float* chain,
                                          int depth, int seq_len, MtpRow* catch_rows, int* catch_tok,
                                          int* catch_hidx) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  if (b >= nseq) return;
  greedy_accept_seq(sr, b, kmax, vmax, vhid, d, chain, depth, seq_len, catch_rows, catch_tok, catch_hidx);
}

}  // namespace lz98
