// Tensor-core int8 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a)
// for R > 8 token rows: y (R x N) = [y +] W x (+ W2 x2).
//
// Every 32-element sub-block dot product of the reference (the exact int32
// it accumulates per 32, src/ops_matmul.c:336-647) is ONE tcgen05.mma of
// kind::i8 with M = 128 weight rows, N = NT token rows, K = 32, issued with
// the accumulator input disabled, so the tensor memory (TMEM) column block
// it writes holds exactly that int32 for every (weight row, token) pair.
// The four sub-blocks of a 128-byte K slice go to four column blocks of one
// TMEM buffer; two buffers alternate so the MMAs of slice i+1 run while the
// epilogue reads slice i.  The reference's float epilogue
// (src/ops_epi.c:983-1023) then runs per (output, token) in K order on the
// CUDA cores, the int32 read back with tcgen05.ld.
//
// Warp roles (320 threads, two CTAs per SM):
//   warps 0-7  epilogue: warp w reads TMEM lanes 32 (w % 4) .. +32 (one
//              weight row per thread) and tokens 8 (w / 4) .. +8, its
//              arithmetic on token pairs with the packed f32x2 operations;
//   warp 8     producer: 2-D TMA loads of each K slice (weight tile 128 x
//              128 B and token tile NT x 128 B, both 128-byte swizzled, the
//              per-32 activation scales and, for gs = 32, the weight
//              scales) into a ring of kUmmaStages stages;
//   warp 9     MMA issuer (one thread), also the TMEM allocator warp.
// Barriers: full[s] (TMA bytes landed), empty[s] (1 MMA commit + 8
// epilogue warps: the stage's tiles and scales are no longer read),
// tfull[b] (MMA commit: TMEM buffer b written), tempty[b] (8 epilogue
// warps: buffer b read).  Every wait is bounded (mbar_wait); a wait that
// gives up sets *err, the CTA skips its stores, lets every issued copy and
// MMA finish and frees its TMEM before exiting.
#pragma once
#include "lz98_kernels.cuh"

namespace lz98 {

constexpr int kUmmaStages = 4;
constexpr int kUmmaM = 128;          // weight rows per CTA (MMA M, TMEM lanes)
constexpr int kUmmaThreads = 320;

// Shared-memory descriptor of a K-major operand tile written by a 2-D TMA
// load with the 128-byte swizzle: 8-row x 128-byte atoms 1024 bytes apart
// (stride byte offset 1024), leading byte offset unused (1), descriptor
// version 1, layout type 2 (128-byte swizzle).  The tile base is 1024-byte
// aligned; sub-block j of the slice starts 32 j bytes in.
LZ_HD uint64_t umma_desc_sw128(uint32_t saddr) {
  const uint64_t lo = (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16);
  const uint64_t hi = (uint64_t)(1024 >> 4) | ((uint64_t)1 << 14) | ((uint64_t)2 << 29);
  return lo | (hi << 32);
}

// Instruction descriptor of kind::i8: D s32, A and B signed int8, both
// K-major, N = n, M = 128.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kUmmaM >> 4) << 24);
}

LZ_HD void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
LZ_HD void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
LZ_HD void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LZ_HD void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LZ_HD void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (TMEM) = A x B with the accumulator input disabled: the exact int32
// sums of one 32-wide K step.
LZ_HD void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(0)
      : "memory");
}
// Arrive (once) on the barrier when every MMA this thread issued so far
// has completed.
LZ_HD void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Four 8-column TMEM reads of this warp's 32 lanes (columns c + step j,
// j = 0..3: the thread's 8 tokens of the four sub-blocks of a K slice) and
// the wait for them, in one statement so that no register is read before
// the wait.
LZ_HD void tmem_ld_4x8(uint32_t taddr, uint32_t step, int (&v)[4][8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%32];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%33];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%34];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%24,%25,%26,%27,%28,%29,%30,%31}, [%35];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(v[0][0]), "=r"(v[0][1]), "=r"(v[0][2]), "=r"(v[0][3]), "=r"(v[0][4]), "=r"(v[0][5]), "=r"(v[0][6]),
        "=r"(v[0][7]), "=r"(v[1][0]), "=r"(v[1][1]), "=r"(v[1][2]), "=r"(v[1][3]), "=r"(v[1][4]), "=r"(v[1][5]),
        "=r"(v[1][6]), "=r"(v[1][7]), "=r"(v[2][0]), "=r"(v[2][1]), "=r"(v[2][2]), "=r"(v[2][3]), "=r"(v[2][4]),
        "=r"(v[2][5]), "=r"(v[2][6]), "=r"(v[2][7]), "=r"(v[3][0]), "=r"(v[3][1]), "=r"(v[3][2]), "=r"(v[3][3]),
        "=r"(v[3][4]), "=r"(v[3][5]), "=r"(v[3][6]), "=r"(v[3][7])
      : "r"(taddr), "r"(taddr + step), "r"(taddr + 2u * step), "r"(taddr + 3u * step)
      : "memory");
}

// Two-lane float arithmetic of the epilogue: with LZ98_PACKED_F32X2 = 1
// the packed f32x2 operations, else the scalar __fadd_rn / __fmul_rn lane
// by lane (the default).
#ifndef LZ98_PACKED_F32X2
#define LZ98_PACKED_F32X2 0
#endif
LZ_HD float2 add2(float2 a, float2 b) {
#if LZ98_PACKED_F32X2
  return __fadd2_rn(a, b);
#else
  return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
#endif
}
LZ_HD float2 mul2(float2 a, float2 b) {
#if LZ98_PACKED_F32X2
  return __fmul2_rn(a, b);
#else
  return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
#endif
}

// Exact int32 -> float of two sub-block sums (|v| < 2^22: the 1.5 2^23
// magic add, then the magic subtracted; x - c and x + (-c) round alike).
LZ_HD float2 i2f_small2(int v0, int v1) {
  return add2(make_float2(__int_as_float(0x4B400000 + v0), __int_as_float(0x4B400000 + v1)),
              make_float2(-12582912.0f, -12582912.0f));
}

// Stage layout of the UMMA GEMM with NT token rows per CTA.
template <int NT, bool RB1>
struct UmmaTile {
  static constexpr int A = kUmmaM * 128;          // weight tile (1024-byte aligned)
  static constexpr int B = NT * 128;              // token tile (NT % 8 == 0: 1024-byte aligned)
  static constexpr int X = NT * 16;               // activation scales, 4 per token row
  static constexpr int W = RB1 ? kUmmaM * 16 : 0; // weight scales (gs = 32)
  static constexpr int TILES = A + B;
  static constexpr int SMALL = X + W;
  static constexpr uint32_t TCOLS = 8 * NT;       // two buffers of four NT-column blocks
  // 1024 alignment slack, the stages, 2 S + 4 barriers, the TMEM address
  static constexpr size_t smem() {
    return 1024 + (size_t)kUmmaStages * (TILES + SMALL) + (2 * kUmmaStages + 4) * 8 + 16;
  }
};

// The float epilogue state of this thread: one weight row, 8 tokens as 4
// pairs (packed f32x2 arithmetic: each lane of a pair rounds as the scalar
// operation does, so the reference's order is kept per token).
template <bool RB1>
struct UmmaAcc {
  float2 a[RB1 ? 4 : 2][4];   // [accumulator][token pair]
};

template <int NT, int GM>
__global__ void __launch_bounds__(kUmmaThreads, 2) gemm_q8_umma_kernel(const __grid_constant__ GemmTmaArgs p) {
  constexpr bool RB1 = GM == 0;
  using T = UmmaTile<NT, RB1>;
  constexpr int S = kUmmaStages;
  static_assert(NT == 16, "epilogue warps take 8 tokens each, two warps per lane quarter");
  extern __shared__ uint8_t umma_smem[];
  const uint32_t raw = smem_u32(umma_smem);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t small = base + S * T::TILES;
  const uint32_t bars = small + S * T::SMALL;   // full[s] +8s, empty[s] +8(S+s), tfull[b] +8(2S+b), tempty[b] +8(2S+2+b)
  const uint32_t taddr_slot = bars + (2 * S + 4) * 8;
  const uint8_t* gsmall = umma_smem + (small - raw);
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kUmmaM, r0 = blockIdx.y * NT;
  const int nsb = p.K >> 5, nsb2 = p.dual ? p.K2 >> 5 : 0;
  const int it1 = nsb / kTmaSub, nit = it1 + nsb2 / kTmaSub;
  if (warp == 8 && lane == 0 && blockIdx.y == 0) {   // weights stream into L2 before the wait
    const int rows = min(kUmmaM, p.N - n0);
    prefetch_l2(p.W + (size_t)n0 * p.K, (size_t)rows * p.K);
    if (p.dual) prefetch_l2(p.W2 + (size_t)n0 * p.K2, (size_t)rows * p.K2);
  }
  pdl_wait();
  if (threadIdx.x == 256) {
    for (int s = 0; s < S; s++) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (S + s), 9);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(bars + 8 * (2 * S + b), 1);
      mbar_init(bars + 8 * (2 * S + 2 + b), 8);
    }
    mbar_fence_init();
  }
  if (warp == 9) tmem_alloc(taddr_slot, T::TCOLS);   // the whole warp; address into shared memory
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(umma_smem + (taddr_slot - raw));
  bool ok = true;
  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      const bool skip0 = g_dbg_skip_stage != 0;   // test hook: stage 0 is never filled
      for (; it < nit; it++) {
        const int stg = it % S;
        if (it >= S && !mbar_wait(bars + 8 * (S + stg), (it / S - 1) & 1)) {
          ok = false;
          break;
        }
        fence_proxy_async_smem();
        if (skip0 && it == 0) continue;
        const bool two = it >= it1;
        const int c = two ? it - it1 : it;
        const uint32_t full = bars + 8 * stg, tile = base + stg * T::TILES, sm = small + stg * T::SMALL;
        mbar_expect_tx(full, T::A + T::B + T::X + T::W);
        tma_load_2d(tile, two ? &p.b2 : &p.b, c * 128, n0, full);           // weights: the MMA's A
        tma_load_2d(tile + T::A, two ? &p.a2 : &p.a, c * 128, r0, full);    // tokens: the MMA's B
        tma_load_2d(sm, two ? &p.x2 : &p.x, c * kTmaSub, r0, full);
        if (RB1) tma_load_2d(sm + T::X, two ? &p.w2 : &p.w, c * kTmaSub, n0, full);
      }
      if (!ok) atomicExch(p.err, 1);
      // every copy issued lands before the block exits
      for (int j = max(0, it - S); j < it; j++)
        if (!(skip0 && j == 0)) mbar_wait(bars + 8 * (j % S), (j / S) & 1);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(NT);
      int it = 0;
      for (; it < nit && ok; it++) {
        const int stg = it % S, buf = it & 1;
        if (!mbar_wait(bars + 8 * stg, (it / S) & 1)) { ok = false; break; }
        if (it >= 2 && !mbar_wait(bars + 8 * (2 * S + 2 + buf), ((it >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tile = base + stg * T::TILES;
        const uint64_t da = umma_desc_sw128(tile), db = umma_desc_sw128(tile + T::A);
#pragma unroll
        for (int j = 0; j < kTmaSub; j++)
          umma_i8(tmem + (uint32_t)(buf * 4 * NT + j * NT), da + (uint64_t)(2 * j), db + (uint64_t)(2 * j), idesc);
        umma_commit(bars + 8 * (2 * S + buf));   // the buffer is written
        umma_commit(bars + 8 * (S + stg));       // the stage's tiles are read
      }
      if (!ok) atomicExch(p.err, 1);
      // the last MMAs have completed before TMEM is freed
      if (it > 0) mbar_wait(bars + 8 * (2 * S + ((it - 1) & 1)), ((it - 1) >> 1) & 1);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3, half = warp >> 2;
    const int row = q * 32 + lane;                  // weight row inside the tile
    const int n = min(n0 + row, p.N - 1);
    UmmaAcc<RB1> st;
    float2 v[4];
    int gcnt = 0, gidx = 0;
    float wrow = 0.0f;
    const float2 zero2 = make_float2(0.0f, 0.0f);
    for (int it = 0; it < nit; it++) {
      const bool two = it >= it1;
      if (it == 0 || it == it1) {
        // a product starts: zero its reduction state (src/ops_epi.c:983-1023)
#pragma unroll
        for (int j = 0; j < (RB1 ? 4 : 2); j++)
#pragma unroll
          for (int cp = 0; cp < 4; cp++) st.a[j][cp] = zero2;
        gcnt = gidx = 0;
        if (GM == 1) wrow = __ldg((two ? p.ws2 : p.ws) + n);
      }
      const int stg = it % S, buf = it & 1;
      if (!mbar_wait(bars + 8 * (2 * S + buf), (it >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const int K = two ? p.K2 : p.K, gs = two ? p.gs2 : p.gs;
      const int rb = gs >> 5, ng = K / gs, c0 = (two ? it - it1 : it) * kTmaSub;
      int d[4][8];
      tmem_ld_4x8(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 4 * NT + half * 8), (uint32_t)NT, d);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8 * (2 * S + 2 + buf));   // TMEM buffer read
      // the stage's scales (its TMA bytes have landed: the MMAs ran on
      // them; the wait only orders this thread's shared-memory reads)
      if (!mbar_wait(bars + 8 * stg, (it / S) & 1)) { ok = false; break; }
      const float* xsm = reinterpret_cast<const float*>(gsmall + stg * T::SMALL);
      float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (RB1) wv = *reinterpret_cast<const float4*>(xsm + NT * 4 + row * 4);
      float2 xv[8];   // the activation scales of sub-blocks j, j + 1 for the 8 tokens
#pragma unroll
      for (int j = 0; j < kTmaSub; j++) {
        if ((j & 1) == 0) {
#pragma unroll
          for (int c = 0; c < 8; c++) xv[c] = *reinterpret_cast<const float2*>(xsm + (half * 8 + c) * 4 + j);   // broadcast
          if (j == 2) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bars + 8 * (S + stg));   // the stage's scales are in registers
          }
        }
        const int s = c0 + j;
        bool gend = false;
        float wg = 0.0f;
        if (GM == 1) {
          gend = s == (K >> 5) - 1;
          wg = wrow;
        } else if (GM == 2) {
          gend = ++gcnt == rb;
          if (gend) {
            gcnt = 0;
            wg = __ldg((two ? p.ws2 : p.ws) + (size_t)n * ng + gidx);
            gidx++;
          }
        } else {
          wg = f4_at(wv, j);
        }
        const float2 wg2 = make_float2(wg, wg);
#pragma unroll
        for (int cp = 0; cp < 4; cp++) {
          const float2 a = i2f_small2(d[j][2 * cp], d[j][2 * cp + 1]);
          const float2 xs2 = (j & 1) ? make_float2(xv[2 * cp].y, xv[2 * cp + 1].y)
                                     : make_float2(xv[2 * cp].x, xv[2 * cp + 1].x);
          if (!RB1) {
            st.a[0][cp] = add2(st.a[0][cp], mul2(a, xs2));
            if (gend) {
              st.a[1][cp] = add2(st.a[1][cp], mul2(st.a[0][cp], wg2));
              st.a[0][cp] = zero2;
            }
          } else {
            // K % 128 == 0: the interleaved accumulator of sub-block s is s & 3 == j
            st.a[j][cp] = add2(st.a[j][cp], mul2(a, mul2(xs2, wg2)));
          }
        }
      }
      if (it == it1 - 1 || it == nit - 1) {
        // a product ends: its value per token (the second is added to the first)
#pragma unroll
        for (int cp = 0; cp < 4; cp++) {
          const float2 r = RB1 ? add2(add2(st.a[0][cp], st.a[2][cp]), add2(st.a[1][cp], st.a[3][cp]))
                               : st.a[1][cp];
          v[cp] = it == it1 - 1 ? r : add2(v[cp], r);
        }
      }
    }
    if (!ok) {
      atomicExch(p.err, 1);
    } else if (n0 + row < p.N) {
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const int r = r0 + half * 8 + c;
        const float vc = (c & 1) ? v[c >> 1].y : v[c >> 1].x;
        if (r < p.R) {
          float* yp = p.y + (size_t)r * p.ldy + n0 + row;
          *yp = p.mode == 1 ? __fadd_rn(*yp, vc) : vc;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, T::TCOLS);
    tmem_relinquish();
  }
}

}  // namespace lz98
