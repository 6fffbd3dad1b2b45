// Head-slab packing for DeepSpeed-Ulysses resharding.
//
// The tokens->heads all-to-all of vidax's sequence_parallel_self_attention
// (jax.lax.all_to_all(x, split_axis=2, concat_axis=1, tiled=True),
// src/vidax/core/attention.py:379-381) sends head group g of every local
// token to rank g. With one NCCL all-to-all over equal contiguous chunks,
// chunk g of the send buffer must hold exactly that group:
//
//   pack:   src (S_loc, H, D) strided rows of one batch item
//           -> dst (G, S_loc, Hg, D) contiguous, h = g*Hg + hg
//
// where Hg = ceil(H / G); heads h >= H (padding when H % G != 0) are written
// as zeros. A sub-group form packs heads head_offset + g*group_stride + i,
// i < Hg, of each group (one slice of every rank's head group), so the
// exchange can be split into pipelined pieces. The receiving rank then holds (G_src, S_loc, Hg, D) = (S, Hg, D)
// in natural token order, which the attention kernel reads directly.
//
// The inverse (heads->tokens, attention.py:388) unpacks the received
// (G_src, S_loc, Hg, D) buffer back to strided (S_loc, H, D) rows, dropping
// padded heads.
//
// Both are pure 16-byte vector copies (HBM-bound); up to three tensors
// (q, k, v) move in one launch.
//
// Peer forms (kPeer): the exchange itself, done by these kernels' stores and
// loads over NVLink into / from the other ranks' memory (mapped into this
// process by CUDA IPC), so the pack and the all-to-all are one pass:
//   pack:   group g's chunk goes straight to peer[t][g], the slot rank g
//           keeps for this rank's chunk in its receive slab;
//   unpack: group g's chunk is read straight from peer[t][g], the slot of
//           this rank's tokens in rank g's attention output.
#pragma once

#include "sm100_common.cuh"

namespace vx {
namespace ulysses {

constexpr int kMaxPeerGroups = 8;  // one NVLink / NVSwitch domain

struct PackParams {
  const uint4* src[3];
  uint4* dst[3];
  long long s_stride[3];  // strided side: token stride in 16-byte vectors
  long long h_stride[3];  // strided side: head stride in 16-byte vectors
  int num_tensors;
  int seq;       // S_loc
  int heads;     // H (real heads on the strided side)
  int hg;        // heads per group on the packed side
  int groups;    // G
  int vpd_log2;  // log2(D / 8): 16-byte vectors per head row
  int group_stride;  // strided-side heads between consecutive groups
  int head_offset;   // strided head of group 0's first packed head
  int group_valid;   // packed heads per group that map to real heads
  uint4* peer[3][kMaxPeerGroups];  // kPeer: per group, the packed chunk's remote address
};

// grid = (x: chunks of the (s, hg, d) plane of one group, y: group, z: tensor).
// Each thread moves one 16-byte vector; one integer division per vector.
template <bool kPack, bool kPeer = false>
__global__ void __launch_bounds__(256) head_slab_kernel(const __grid_constant__ PackParams p) {
  const int t = blockIdx.z;
  const int g = blockIdx.y;
  const int row_vecs = p.hg << p.vpd_log2;  // vectors per packed (g, s) row
  const long long plane = static_cast<long long>(p.seq) * row_vecs;
  // the packed chunk of group g: this rank's slab (offset g * plane) or, in
  // the peer forms, its remote slot (offset 0 from the peer address)
  const long long packed_base = kPeer ? 0 : static_cast<long long>(g) * plane;
  const uint4* __restrict__ src = (kPeer && !kPack) ? p.peer[t][g] : p.src[t];
  uint4* __restrict__ dst = (kPeer && kPack) ? p.peer[t][g] : p.dst[t];
  const long long ss = p.s_stride[t], hs = p.h_stride[t];
  const int dmask = (1 << p.vpd_log2) - 1;
  for (long long idx = blockIdx.x * 256LL + threadIdx.x; idx < plane;
       idx += static_cast<long long>(gridDim.x) * 256) {
    const int s = static_cast<int>(idx / row_vecs);
    const int c = static_cast<int>(idx - static_cast<long long>(s) * row_vecs);
    const int i = c >> p.vpd_log2;
    const int h = p.head_offset + g * p.group_stride + i;
    const bool valid = i < p.group_valid && h < p.heads;
    const long long strided = s * ss + h * hs + (c & dmask);
    if (kPack) {
      uint4 val = make_uint4(0, 0, 0, 0);
      if (valid) val = __ldg(src + strided);
      dst[packed_base + idx] = val;
    } else {
      if (valid) dst[strided] = __ldg(src + packed_base + idx);
    }
  }
}

}  // namespace ulysses
}  // namespace vx
