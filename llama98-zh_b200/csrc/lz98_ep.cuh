// Expert parallelism: the routed experts of every MoE layer split over the
// ranks of a communicator (rank r owns experts [r epr, (r + 1) epr)), one
// process per GPU, each with its own sequences.  Per layer, after the local
// router (src/ops_moe.c:12-163):
//   1. ep_pack: every (token, expert) pair of this rank goes to the slot
//      buffer of the rank owning its expert, in pair order (a stable slot
//      per destination): the pair's per-32 quantised latent row and scales,
//      the owner-local expert and the pair index;
//   2. the buffers are exchanged (NCCL send/recv to every peer);
//   3. ep_unpack: the pairs received from every rank (this rank's own
//      included) are gathered into one list, source rank by source rank,
//      and run through the grouped expert kernels as pairs of one row each;
//   4. ep_reply: every pair's latent output row goes back to the slot it
//      came from; the rows are exchanged back;
//   5. ep_combine: each token row sums its pairs' rows with its routing
//      weights in selection order (src/forward_moe.c:198-199) - the float
//      operations of the single-GPU combine, on the same values.
// Slot buffer of one peer: a 16-byte header (the pair count) then cap slots
// of slot_bytes: latent int8 | latent/32 f32 scales | expert | pair, padded
// to 16 bytes.
#pragma once
#include "lz98_kernels.cuh"

namespace lz98 {

constexpr int kEpMaxWorld = 8;

struct EpBuf {
  uint8_t* send;           // [world][buf_bytes]
  uint8_t* recv;           // [world][buf_bytes] (this rank's own slot unused: read from send)
  size_t slot_bytes, buf_bytes;
  int cap, latent, world, rank;
};

LZ_HD uint8_t* ep_slot(const EpBuf& b, uint8_t* base, int peer, int i) {
  return base + (size_t)peer * b.buf_bytes + 16 + (size_t)i * b.slot_bytes;
}

// One block of 1024 threads: the stable slot of every pair in its
// destination's buffer (pairs in index order), the slot contents, and
// per destination the count in the header.  pair_dest / pair_slot record
// where each pair's answer will come back (-1: no expert).
__global__ void __launch_bounds__(1024) ep_pack_kernel(const int* __restrict__ pair_e, int P, int topk, int epr,
                                                       const int8_t* __restrict__ latq, const float* __restrict__ lats,
                                                       EpBuf b, int* pair_dest, int* pair_slot) {
  pdl_trigger();
  pdl_wait();
  __shared__ int base[kEpMaxWorld];
  __shared__ int wcnt[32][kEpMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < b.world) base[tid] = 0;
  __syncthreads();
  const int ng = b.latent / 32;
  for (int c0 = 0; c0 < P; c0 += 1024) {
    const int p = c0 + tid;
    int d = -1;
    if (p < P) {
      const int e = pair_e[p];
      if (e >= 0) d = e / epr;
    }
    int mine = 0;
    for (int v = 0; v < b.world; v++) {
      const unsigned bal = __ballot_sync(0xffffffffu, d == v);
      if (lane == 0) wcnt[warp][v] = __popc(bal);
      if (d == v) mine = __popc(bal & ((1u << lane) - 1u));
    }
    __syncthreads();
    if (tid < b.world) {
      int run = base[tid];
      for (int w = 0; w < 32; w++) {
        const int t = wcnt[w][tid];
        wcnt[w][tid] = run;
        run += t;
      }
      base[tid] = run;
    }
    __syncthreads();
    if (p < P) {
      pair_dest[p] = d;
      pair_slot[p] = d >= 0 ? wcnt[warp][d] + mine : -1;
    }
    if (d >= 0) {
      const int slot = wcnt[warp][d] + mine;
      uint8_t* dst = ep_slot(b, b.send, d, slot);
      const int r = p / topk;
      const int4* sq = reinterpret_cast<const int4*>(latq + (size_t)r * b.latent);
      int4* dq = reinterpret_cast<int4*>(dst);
      for (int i = 0; i < b.latent / 16; i++) dq[i] = sq[i];
      float* ds = reinterpret_cast<float*>(dst + b.latent);
      for (int i = 0; i < ng; i++) ds[i] = lats[(size_t)r * ng + i];
      int* di = reinterpret_cast<int*>(ds + ng);
      di[0] = pair_e[p] - d * epr;
      di[1] = p;
    }
    __syncthreads();
  }
  if (tid < b.world) *reinterpret_cast<int*>(b.send + (size_t)tid * b.buf_bytes) = base[tid];
}

// One block of 1024 threads: the pairs received from every source rank,
// source by source, gathered into rows j of latq_ep / lats_ep with their
// owner-local expert (-1 past the total), source and slot.
__global__ void __launch_bounds__(1024) ep_unpack_kernel(EpBuf b, int8_t* latq_ep, float* lats_ep, int* ep_expert,
                                                         int* ep_src, int* ep_slot_of, int* total_out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int off[kEpMaxWorld + 1];
  if (threadIdx.x == 0) {
    int run = 0;
    for (int s = 0; s < b.world; s++) {
      off[s] = run;
      const uint8_t* buf = (s == b.rank ? b.send : b.recv) + (size_t)s * b.buf_bytes;
      run += min(*reinterpret_cast<const int*>(buf), b.cap);
    }
    off[b.world] = run;
    *total_out = run;
  }
  __syncthreads();
  const int total = off[b.world], ng = b.latent / 32;
  for (int j = threadIdx.x; j < b.world * b.cap; j += blockDim.x) {
    if (j >= total) {
      ep_expert[j] = -1;
      continue;
    }
    int s = 0;
    while (j >= off[s + 1]) s++;
    const int i = j - off[s];
    const uint8_t* src = ep_slot(b, s == b.rank ? b.send : b.recv, s, i);
    const int4* sq = reinterpret_cast<const int4*>(src);
    int4* dq = reinterpret_cast<int4*>(latq_ep + (size_t)j * b.latent);
    for (int k = 0; k < b.latent / 16; k++) dq[k] = sq[k];
    const float* ss = reinterpret_cast<const float*>(src + b.latent);
    for (int k = 0; k < ng; k++) lats_ep[(size_t)j * ng + k] = ss[k];
    const int* si = reinterpret_cast<const int*>(ss + ng);
    ep_expert[j] = si[0];
    ep_src[j] = s;
    ep_slot_of[j] = i;
  }
}

// Block j (< the received total): pair j's latent output row to the slot
// it came from - this rank's own pairs straight into the reply buffer,
// the others into the send-back buffer of their source.
__global__ void ep_reply_kernel(const float* __restrict__ h2_ep, const int* __restrict__ ep_src,
                                const int* __restrict__ ep_slot_of, const int* __restrict__ total, int latent, int cap,
                                int rank, float* sendback, float* recvback) {
  pdl_trigger();
  pdl_wait();
  const int j = blockIdx.x;
  if (j >= *total) return;
  const int s = ep_src[j];
  float* dst = (s == rank ? recvback : sendback) + ((size_t)s * cap + ep_slot_of[j]) * latent;
  const float* src = h2_ep + (size_t)j * latent;
  for (int i = threadIdx.x; i < latent; i += blockDim.x) dst[i] = src[i];
}

// lat_y of one token row = sum over its selected experts, in selection
// order, of w * (the expert's latent output row, returned by its owner),
// quantised per 32 (src/forward_moe.c:198-199): the operations of
// moe_combine_kernel.
__global__ void ep_combine_kernel(const int* __restrict__ pair_e, const float* __restrict__ pair_w,
                                  const int* __restrict__ pair_dest, const int* __restrict__ pair_slot, int topk,
                                  const float* __restrict__ recvback, int cap, int latent, int8_t* yq, float* ys) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int g = warp; g < latent / 32; g += blockDim.x >> 5) {
    const int i = g * 32 + lane;
    float acc = 0.0f;
    for (int t = 0; t < topk; t++) {
      const int pp = r * topk + t;
      if (pair_e[pp] < 0) continue;
      const float h = recvback[((size_t)pair_dest[pp] * cap + pair_slot[pp]) * latent + i];
      acc = __fadd_rn(acc, __fmul_rn(pair_w[pp], h));
    }
    yq[(size_t)r * latent + i] = warp_quant32(acc, &ys[(size_t)r * (latent / 32) + g]);
  }
}

}  // namespace lz98
