// Fused elementwise glue of the DiT block (HBM-bound, one pass each).
//
// vidax's WanDiTBlock (src/vidax/models/wan/wan2_1/dit.py:100-156) keeps the
// residual stream x in float32 and, around every sub-layer, runs
//   y = bf16(LayerNorm(x) [* w + b] * (1 + scale) + shift)      (:106-108, :119-122, :129-131)
//   x = x + float(sub_layer_out) * gate                         (:113, :123-127, :155)
// As separate framework ops that is 5-7 full passes over a float32 tensor
// per use; here each is one pass:
//
// ln_modulate_kernel: one warp per row. Pass 1 accumulates sum(x) and
//   sum(x^2) in float32 (flax's LayerNorm statistics: var = E[x^2] - E[x]^2,
//   clamped at 0); pass 2 re-reads the row (L1 / L2) and writes bf16.
//   Optional per-feature affine (w, b) and per-batch-item modulation
//   (scale, shift of shape (batches, dim)).
// gated_residual_kernel: x[r] += float(y[r]) * gate[batch(r)] (gate optional),
//   8 features per thread and iteration (16-byte bf16 / 32-byte float loads).
#pragma once

#include <cuda_bf16.h>

#include "sm100_common.cuh"

namespace vx {
namespace glue {

struct LnParams {
  const float* x;        // (rows, dim)
  __nv_bfloat16* y;      // (rows, dim)
  const float* w;        // (dim) or NULL
  const float* b;        // (dim) or NULL
  const float* scale;    // (batches, dim) or NULL
  const float* shift;    // (batches, dim) or NULL
  long long rows;
  int dim;               // multiple of 4
  int rows_per_batch;
  float eps;
};

__global__ void __launch_bounds__(256) ln_modulate_kernel(const __grid_constant__ LnParams p) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int lane = threadIdx.x & 31;
  const float4* x4 = reinterpret_cast<const float4*>(p.x + row * p.dim);
  const int n4 = p.dim >> 2;
  float s = 0.f, s2 = 0.f;
  for (int i = lane; i < n4; i += 32) {
    const float4 v = x4[i];
    s += (v.x + v.y) + (v.z + v.w);
    s2 = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s2))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  const float inv_n = 1.0f / static_cast<float>(p.dim);
  const float mean = s * inv_n;
  const float var = fmaxf(s2 * inv_n - mean * mean, 0.f);
  const float rstd = rsqrtf(var + p.eps);
  const long long bi = row / p.rows_per_batch;
  const float4* sc4 = p.scale ? reinterpret_cast<const float4*>(p.scale + bi * p.dim) : nullptr;
  const float4* sh4 = p.shift ? reinterpret_cast<const float4*>(p.shift + bi * p.dim) : nullptr;
  const float4* w4 = p.w ? reinterpret_cast<const float4*>(p.w) : nullptr;
  const float4* b4 = p.b ? reinterpret_cast<const float4*>(p.b) : nullptr;
  uint2* y2 = reinterpret_cast<uint2*>(p.y + row * p.dim);
  for (int i = lane; i < n4; i += 32) {
    const float4 v = x4[i];
    float f[4] = {(v.x - mean) * rstd, (v.y - mean) * rstd, (v.z - mean) * rstd,
                  (v.w - mean) * rstd};
    if (w4) {
      const float4 ww = __ldg(w4 + i), bb = __ldg(b4 + i);
      f[0] = fmaf(f[0], ww.x, bb.x);
      f[1] = fmaf(f[1], ww.y, bb.y);
      f[2] = fmaf(f[2], ww.z, bb.z);
      f[3] = fmaf(f[3], ww.w, bb.w);
    }
    if (sc4) {
      const float4 c = __ldg(sc4 + i), d = __ldg(sh4 + i);
      f[0] = fmaf(f[0], 1.f + c.x, d.x);
      f[1] = fmaf(f[1], 1.f + c.y, d.y);
      f[2] = fmaf(f[2], 1.f + c.z, d.z);
      f[3] = fmaf(f[3], 1.f + c.w, d.w);
    }
    y2[i] = make_uint2(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]));
  }
}

struct ResidualParams {
  float* x;                   // (rows, dim), updated in place
  const __nv_bfloat16* y;     // (rows, dim)
  const float* gate;          // (batches, dim) or NULL
  long long rows;
  int dim;                    // multiple of 8
  int rows_per_batch;
};

__global__ void __launch_bounds__(256) gated_residual_kernel(const __grid_constant__ ResidualParams p) {
  const int n8 = p.dim >> 3;
  const long long total = p.rows * n8;
  for (long long idx = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * 256) {
    const long long row = idx / n8;
    const int c = static_cast<int>(idx - row * n8);
    float4* xr = reinterpret_cast<float4*>(p.x + row * p.dim) + 2 * c;
    const uint4 yv = __ldg(reinterpret_cast<const uint4*>(p.y + row * p.dim) + c);
    const uint32_t w[4] = {yv.x, yv.y, yv.z, yv.w};
    float f[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      f[2 * k] = __uint_as_float(w[k] << 16);
      f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
    if (p.gate) {
      const float4* g4 = reinterpret_cast<const float4*>(p.gate + (row / p.rows_per_batch) * p.dim) + 2 * c;
      const float4 g0 = __ldg(g4), g1 = __ldg(g4 + 1);
      f[0] *= g0.x; f[1] *= g0.y; f[2] *= g0.z; f[3] *= g0.w;
      f[4] *= g1.x; f[5] *= g1.y; f[6] *= g1.z; f[7] *= g1.w;
    }
    float4 a = xr[0], b = xr[1];
    a.x += f[0]; a.y += f[1]; a.z += f[2]; a.w += f[3];
    b.x += f[4]; b.y += f[5]; b.z += f[6]; b.w += f[7];
    xr[0] = a;
    xr[1] = b;
  }
}

}  // namespace glue
}  // namespace vx
