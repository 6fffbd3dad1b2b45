// Fused pre-attention step: QK RMSNorm + 3-D RoPE + head-slab pack.
//
// What it replaces (vidax, per attention layer, after the q/k/v Dense):
//
//   q = RMSNorm(dim)(q); k = RMSNorm(dim)(k)         attention.py:149-162,
//                                                    wan/common/dit_layers.py:137-143
//   q, k, v = reshape(B, S, H, D)                    dit_layers.py:145-147
//   q = apply_rope3d(q, freqs); k = ...              rope3d.py:89-111, dit_layers.py:148-149
//   all_to_all packing of sequence_parallel_self_attention (attention.py:379-381)
//
// i.e. four separate HBM passes over q and k (norm, reshape-copy, RoPE,
// all-to-all send layout) become one: every token row is read once, and the
// normalised, rotated heads are written straight into the Ulysses send slabs
// of every pipelined slice. HunyuanVideo / LTX-2.5 normalise per head
// (RMSNorm(head_dim), hunyuan_video/common/dit_layers.py:358, ltx2_5/
// diffusion_vae.py:263) -- the same kernel with per_head = 1.
//
// Arithmetic (bit-exact with the reference's float32 formulas given the same
// mean square; only the summation order of sum(x^2) is the kernel's own):
//   var   = sum(x^2) / cols                     (float32)
//   n     = bf16(x * (1 / sqrt(var + eps)))      IEEE sqrt and divide
//   y     = bf16(n * bf16(w))                    bf16 x bf16 product
//   y     = bf16(y * post_scale)                 only when post_scale != 1
//   rope  : (a, b) -> (bf16(a c - b s), bf16(b c + a s)) on adjacent pairs,
//           products and sums each rounded in float32 (no FMA contraction).
//
// Layout: one warp per (token row, tensor). Lane l holds the 16-byte vectors
// v = 32 i + l of the row (8 bf16 each), so a head of D elements sits in
// D/8 consecutive lanes and per-head sums reduce with xor shuffles inside that
// lane segment. Output per tensor and batch item, slice by slice:
//   [slice j][group g][token s][head i < slice_heads[j]][d]
// with zero heads past H (padding when H % G != 0).
#pragma once

#include <cuda_bf16.h>

#include "sm100_common.cuh"

namespace vx {
namespace prologue {

constexpr int kMaxSlices = 8;
constexpr int kWarpsPerCta = 4;

struct NormRopeParams {
  const uint4* src[3];
  uint4* dst[3];
  long long b_stride[3], s_stride[3], h_stride[3];  // source strides in 16-byte vectors
  const float* weight[3];                           // NULL = no norm
  float post_scale[3];
  const float* cos;  // (seq, D/2) per-token tables
  const float* sin;
  long long rope_stride;  // floats between consecutive tokens' tables
  int rope_mask;          // bit t: rotate tensor t
  int num_tensors, batch, seq, heads;
  int vpd_log2;  // log2(D / 8)
  int per_head;  // norm over each head's D features instead of the whole row
  float eps;
  float cols;    // features per norm group (float, divisor of the mean)
  int groups, hg;
  int num_slices;
  int slice_off[kMaxSlices + 1];  // prefix sums of the slices' heads; slice_off[num_slices] = hg
  long long item_vecs;            // packed 16-byte vectors per tensor and batch item
};

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

__device__ __forceinline__ void unpack8(const uint4& x, float f[8]) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = bf16_lo(w[k]);
    f[2 * k + 1] = bf16_hi(w[k]);
  }
}

__device__ __forceinline__ uint4 pack8(const float f[8]) {
  return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

// Packed 16-byte vector index (within one batch item) of head h's vector dv
// of token s.
__device__ __forceinline__ long long packed_index(const NormRopeParams& p, int s, int h, int dv) {
  const int g = h / p.hg;
  const int i = h - g * p.hg;
  int j = 0;
#pragma unroll
  for (int k = 1; k < kMaxSlices; ++k)
    if (k < p.num_slices && i >= p.slice_off[k]) j = k;
  const int off = p.slice_off[j];
  const int hs = p.slice_off[j + 1] - off;
  const long long base = static_cast<long long>(p.groups) * p.seq * off;  // slice start, in head rows
  const long long row = base + (static_cast<long long>(g) * p.seq + s) * hs + (i - off);
  return (row << p.vpd_log2) + dv;
}

// kV: 16-byte vectors held per lane (rows of up to 32 * kV * 8 features).
template <int kV>
__global__ void __launch_bounds__(kWarpsPerCta * 32) norm_rope_pack_kernel(
    const __grid_constant__ NormRopeParams p) {
  const int t = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  if (row >= static_cast<long long>(p.batch) * p.seq) return;
  const int b = static_cast<int>(row / p.seq);
  const int s = static_cast<int>(row - static_cast<long long>(b) * p.seq);
  const int dmask = (1 << p.vpd_log2) - 1;
  const int nvec = p.heads << p.vpd_log2;
  const uint4* __restrict__ src = p.src[t] + b * p.b_stride[t] + s * p.s_stride[t];
  const long long hstr = p.h_stride[t];

  uint4 x[kV];
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    const int v = i * 32 + lane;
    x[i] = make_uint4(0, 0, 0, 0);
    if (v < nvec) x[i] = __ldg(src + (v >> p.vpd_log2) * hstr + (v & dmask));
  }

  const float* __restrict__ w = p.weight[t];
  const float ps = p.post_scale[t];
  const bool rope = (p.rope_mask >> t) & 1;
  if (w != nullptr || ps != 1.0f || rope) {
    float rinv[kV];
    if (w != nullptr) {
      if (!p.per_head) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < kV; ++i) {
          float f[8];
          unpack8(x[i], f);
#pragma unroll
          for (int k = 0; k < 8; ++k) acc = fmaf(f[k], f[k], acc);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        const float var = __fdiv_rn(acc, p.cols);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
#pragma unroll
        for (int i = 0; i < kV; ++i) rinv[i] = r;
      } else {
        const int seg = 1 << p.vpd_log2;  // lanes per head (8, 16 or 32)
#pragma unroll
        for (int i = 0; i < kV; ++i) {
          float f[8];
          unpack8(x[i], f);
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) acc = fmaf(f[k], f[k], acc);
          for (int o = seg >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
          const float var = __fdiv_rn(acc, p.cols);
          rinv[i] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
        }
      }
    }
    const float* __restrict__ cs = p.cos + s * p.rope_stride;
    const float* __restrict__ sn = p.sin + s * p.rope_stride;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int v = i * 32 + lane;
      if (v >= nvec) continue;
      const int dv = v & dmask;
      float f[8];
      unpack8(x[i], f);
      if (w != nullptr) {
        const float* wp = w + (p.per_head ? 0 : (v >> p.vpd_log2) << (p.vpd_log2 + 3)) + dv * 8;
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(wp));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(wp) + 1);
        const float wf[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float n = round_bf16(__fmul_rn(f[k], rinv[i]));
          f[k] = round_bf16(__fmul_rn(n, round_bf16(wf[k])));
        }
      }
      if (ps != 1.0f) {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = round_bf16(__fmul_rn(f[k], ps));
      }
      if (rope) {
        const float4 c = __ldg(reinterpret_cast<const float4*>(cs + dv * 4));
        const float4 sv = __ldg(reinterpret_cast<const float4*>(sn + dv * 4));
        const float cc[4] = {c.x, c.y, c.z, c.w};
        const float ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a = f[2 * k], bb = f[2 * k + 1];
          f[2 * k] = __fsub_rn(__fmul_rn(a, cc[k]), __fmul_rn(bb, ss[k]));
          f[2 * k + 1] = __fadd_rn(__fmul_rn(bb, cc[k]), __fmul_rn(a, ss[k]));
        }
      }
      x[i] = pack8(f);
    }
  }

  uint4* __restrict__ dst = p.dst[t] + b * p.item_vecs;
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    const int v = i * 32 + lane;
    if (v < nvec) dst[packed_index(p, s, v >> p.vpd_log2, v & dmask)] = x[i];
  }
  // zero heads past H (head padding of the last groups)
  const int nvec_all = (p.groups * p.hg) << p.vpd_log2;
  for (int v = nvec + lane; v < nvec_all; v += 32)
    dst[packed_index(p, s, v >> p.vpd_log2, v & dmask)] = make_uint4(0, 0, 0, 0);
}

}  // namespace prologue
}  // namespace vx
