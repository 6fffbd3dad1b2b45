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
// Layout: a persistent CTA (one per SM) streams work items -- R consecutive
// tokens of one tensor -- through a ring of shared-memory stages. Lanes 0-3
// of warp 0 are the producer: in lockstep, each waits for the stage of its
// own item and fills it with untiled bulk copies (one for the R rows when the
// tokens are adjacent in memory, else one per row or per head) plus, for
// rotated tensors, the tokens' cos / sin rows into a table slot of the same
// index (one copy when the cos and sin rows are interleaved per token). Four
// lanes keep four fills in flight per issue round; one thread alone issues
// one copy per ~400 cycles, too few for HBM rates with small rows.
//
// Warps 1..8 are consumers, each owning whole items (item n of the CTA goes to
// warp n % 8; the ring depth is a multiple of 8, so stage n % S is waited on
// by one warp only, one phase at a time). Per row, lane l handles the 16-byte
// vectors v = l + 32 i (8 bf16 each) in rolled loops that read the stage:
// pass 1 sums x^2, pass 2 transforms and stores. A head of D elements is D/8
// consecutive lanes, so per-head sums reduce with xor shuffles inside that
// lane segment. Rolled loops keep the code small (the fully unrolled form
// stalled on instruction fetch). Destination offsets come from a per-CTA head
// table (slice, group and position of every head), built once.
//
// Output per tensor and batch item, slice by slice:
//   [slice j][group g][token s][head i < slice_heads[j]][d]
// with zero heads past H (padding when H % G != 0).
#pragma once

#include <cuda_bf16.h>

#include "sm100_common.cuh"

namespace vx {
namespace prologue {

constexpr int kMaxSlices = 8;
constexpr int kConsumerWarps = 8;
constexpr int kProducerLanes = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 32;      // a multiple of kConsumerWarps
constexpr int kMinStages = 16;      // 8 held by consumers + at least 8 in flight
constexpr int kStageAlign = 128;
constexpr int kTargetStageBytes = 10 * 1024;  // rows per stage: R = max(1, this / row bytes)
constexpr int kMaxRowsPerStage = 8;
constexpr int kMaxHeadSlots = 512;  // groups * ceil(heads / groups)
// Shared memory of one CTA (one CTA per SM): weights, head table, row ring,
// table ring, control.
constexpr int kSmemBudget = 200 * 1024;

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
  int rows_per_stage;             // R
  int blocks;                     // ceil(seq / R) token blocks per batch item
  int items;                      // num_tensors * batch * blocks
  int stages;                     // ring depth, a multiple of kConsumerWarps
  int stage_bytes;                // R rows, rounded up to kStageAlign
  int row_bytes;                  // heads * D * 2
  int table_bytes;                // cos and sin rows of R tokens (R * D * 4), 0 without RoPE
  int contiguous[3];              // 1: heads adjacent, 2: and tokens adjacent (one copy)
  int table_mode;                 // 2: cos|sin interleaved per token, tokens adjacent;
                                  // 1: interleaved per token; 0: separate tables
  int weight_off[3];              // shared-memory offset of tensor t's bf16 weights (-1: none)
  int head_off;                   // shared-memory offset of the head table
  int ring_off;                   // shared-memory offset of the row ring
  int table_off;                  // shared-memory offset of the table ring
  int ctl_off;                    // shared-memory offset of RingControl
};

// Destination of head slot h (h < groups * hg) for token 0 of a batch item,
// and the distance between consecutive tokens, both in 16-byte vectors.
struct HeadSlot {
  long long base;
  long long token_stride;
};

struct RingControl {
  uint64_t full[kMaxStages];   // rows (and tables) of item n landed in stage n % stages
  uint64_t empty[kMaxStages];  // stage n % stages consumed
  int abort_flag;
};

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
// Two floats -> packed bf16x2 (round to nearest even), one conversion.
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
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

__device__ __forceinline__ HeadSlot head_slot(const NormRopeParams& p, int h) {
  const int g = h / p.hg;
  const int i = h - g * p.hg;
  int j = 0;
  for (int k = 1; k < p.num_slices; ++k)
    if (i >= p.slice_off[k]) j = k;
  const int off = p.slice_off[j];
  const int hs = p.slice_off[j + 1] - off;
  // slice j starts at groups * seq * off head rows; group g of it at g * seq * hs
  const long long row0 = static_cast<long long>(p.groups) * p.seq * off +
                         static_cast<long long>(g) * p.seq * hs + (i - off);
  HeadSlot slot;
  slot.base = row0 << p.vpd_log2;
  slot.token_stride = static_cast<long long>(hs) << p.vpd_log2;
  return slot;
}

// item -> tensor t, batch item b, first token s0 and token count
__device__ __forceinline__ void item_coords(const NormRopeParams& p, int item, int& t, int& b,
                                            int& s0, int& count) {
  const int blk = item / p.num_tensors;
  t = item - blk * p.num_tensors;
  b = blk / p.blocks;
  s0 = (blk - b * p.blocks) * p.rows_per_stage;
  count = min(p.rows_per_stage, p.seq - s0);
}

__device__ __forceinline__ float rms_inverse(float sumsq, float cols, float eps) {
  const float var = __fdiv_rn(sumsq, cols);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// A 16-byte vector (8 bf16 = rotation pairs 4 dv .. 4 dv + 3) as packed
// float pairs: e[0] = (x0, x2), e[1] = (x4, x6) hold the pairs' first
// elements, o[0] = (x1, x3), o[1] = (x5, x7) their second elements -- the
// layout f32x2 arithmetic wants for (pair k, pair k+1) at once.
struct Split8 {
  uint64_t e[2], o[2];
};

__device__ __forceinline__ Split8 split8(const uint4& x) {
  Split8 r;
  r.e[0] = f2_pack(bf16_lo(x.x), bf16_lo(x.y));
  r.o[0] = f2_pack(bf16_hi(x.x), bf16_hi(x.y));
  r.e[1] = f2_pack(bf16_lo(x.z), bf16_lo(x.w));
  r.o[1] = f2_pack(bf16_hi(x.z), bf16_hi(x.w));
  return r;
}

// Back to 8 bf16 (round to nearest even).
__device__ __forceinline__ uint4 join8(const Split8& v) {
  float e0, e1, e2, e3, o0, o1, o2, o3;
  f2_unpack(v.e[0], e0, e1);
  f2_unpack(v.o[0], o0, o1);
  f2_unpack(v.e[1], e2, e3);
  f2_unpack(v.o[1], o2, o3);
  return make_uint4(pack2(e0, o0), pack2(e1, o1), pack2(e2, o2), pack2(e3, o3));
}

// sum of squares of the 8 features into a packed accumulator pair
__device__ __forceinline__ uint64_t sumsq8_acc(const uint4& x, uint64_t acc) {
  const Split8 v = split8(x);
  acc = f2_fma(v.e[0], v.e[0], acc);
  acc = f2_fma(v.o[0], v.o[0], acc);
  acc = f2_fma(v.e[1], v.e[1], acc);
  return f2_fma(v.o[1], v.o[1], acc);
}

__device__ __forceinline__ float f2_sum(uint64_t acc) {
  float a, b;
  f2_unpack(acc, a, b);
  return a + b;
}

// n = bf16(x * r), y = bf16(n * w) (bf16 x bf16 products are exact in
// float32: one rounding, as the reference's bf16 multiply); rr = (r, r).
__device__ __forceinline__ uint4 norm8(const uint4& x, uint64_t rr, const uint4& wv) {
  Split8 v = split8(x);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    v.e[k] = f2_mul(v.e[k], rr);
    v.o[k] = f2_mul(v.o[k], rr);
  }
  const uint4 n = join8(v);
  return make_uint4(mul_bf16x2(n.x, wv.x), mul_bf16x2(n.y, wv.y), mul_bf16x2(n.z, wv.z),
                    mul_bf16x2(n.w, wv.w));
}

__device__ __forceinline__ uint4 scale8(const uint4& x, float ps) {
  float f[8];
  unpack8(x, f);
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = __fmul_rn(f[k], ps);
  return pack8(f);
}

// (a, b) -> (a c - b s, b c + a s) on the 4 pairs, every product and sum
// rounded in float32; c = (c0..c3), sn = (s0..s3) of the 4 pairs. Scalar
// __fmul_rn / __fadd_rn / __fsub_rn: the compiler never fuses them into an
// FMA (packed f32x2 multiplies followed by adds were contracted, changing the
// rounding).
__device__ __forceinline__ uint4 rope8(const uint4& x, const float4& c, const float4& sn) {
  float f[8];
  unpack8(x, f);
  const float cc[4] = {c.x, c.y, c.z, c.w};
  const float ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float a = f[2 * k], b = f[2 * k + 1];
    f[2 * k] = __fsub_rn(__fmul_rn(a, cc[k]), __fmul_rn(b, ss[k]));
    f[2 * k + 1] = __fadd_rn(__fmul_rn(b, cc[k]), __fmul_rn(a, ss[k]));
  }
  return pack8(f);
}

// Issues the bulk copies of item `item` into stage `stage` (producer lane).
__device__ __forceinline__ void fill_stage(const NormRopeParams& p, uint8_t* smem, int item,
                                           int stage, uint32_t full, uint64_t policy) {
  int t, b, s0, count;
  item_coords(p, item, t, b, s0, count);
  const bool rope = (p.rope_mask >> t) & 1;
  const uint32_t head_bytes = 16u << p.vpd_log2;  // D bf16
  const uint32_t tok_table = 32u << p.vpd_log2;   // cos + sin of one token: D floats
  mbar_expect_tx(full, count * p.row_bytes + (rope ? count * tok_table : 0));
  const uint32_t dst = smem_u32(smem + p.ring_off + stage * p.stage_bytes);
  const uint4* src = p.src[t] + b * p.b_stride[t] + s0 * p.s_stride[t];
  if (p.contiguous[t] == 2) {
    bulk_load(dst, src, count * p.row_bytes, full, policy);
  } else {
    for (int r = 0; r < count; ++r) {
      const uint4* row = src + r * p.s_stride[t];
      const uint32_t rdst = dst + r * p.row_bytes;
      if (p.contiguous[t] == 1) {
        bulk_load(rdst, row, p.row_bytes, full, policy);
      } else {
        for (int h = 0; h < p.heads; ++h)
          bulk_load(rdst + h * head_bytes, row + h * p.h_stride[t], head_bytes, full, policy);
      }
    }
  }
  if (rope) {
    const uint32_t tdst = smem_u32(smem + p.table_off + stage * p.table_bytes);
    const float* cs = p.cos + s0 * p.rope_stride;
    if (p.table_mode == 2) {
      bulk_load(tdst, cs, count * tok_table, full, policy);
    } else {
      for (int r = 0; r < count; ++r) {
        if (p.table_mode == 1) {
          bulk_load(tdst + r * tok_table, cs + r * p.rope_stride, tok_table, full, policy);
        } else {
          bulk_load(tdst + r * tok_table, cs + r * p.rope_stride, tok_table / 2, full, policy);
          bulk_load(tdst + r * tok_table + tok_table / 2, p.sin + (s0 + r) * p.rope_stride,
                    tok_table / 2, full, policy);
        }
      }
    }
  }
}

// One token row of one tensor: kNorm 0 none, 1 whole row, 2 per head.
template <int kNorm, bool kScale, bool kRope>
__device__ __forceinline__ void process_row(const NormRopeParams& p, const uint4* __restrict__ row,
                                            const float4* __restrict__ tab,
                                            const uint4* __restrict__ w, float ps,
                                            uint4* __restrict__ dst, const HeadSlot* slots,
                                            int s, int lane) {
  const int dmask = (1 << p.vpd_log2) - 1;
  const int nvec = p.heads << p.vpd_log2;
  const int iters = (nvec + 31) >> 5;
  uint64_t rr = 0;
  if (kNorm == 1) {
    uint64_t acc = 0;
#pragma unroll 4
    for (int i = 0; i < iters; ++i) {
      const int v = lane + 32 * i;
      if (v < nvec) acc = sumsq8_acc(row[v], acc);
    }
    float tot = f2_sum(acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    const float r = rms_inverse(tot, p.cols, p.eps);
    rr = f2_pack(r, r);
  }
#pragma unroll 2
  for (int i = 0; i < iters; ++i) {
    const int v = lane + 32 * i;
    const bool valid = v < nvec;
    const int dv = v & dmask;
    uint4 y = valid ? row[v] : make_uint4(0, 0, 0, 0);
    if (kNorm == 2) {
      float a = f2_sum(sumsq8_acc(y, 0));
      for (int o = (dmask + 1) >> 1; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      const float r = rms_inverse(a, p.cols, p.eps);
      rr = f2_pack(r, r);
    }
    if (!valid) continue;
    if (kNorm != 0) y = norm8(y, rr, w[kNorm == 2 ? dv : v]);
    if (kScale) y = scale8(y, ps);
    if (kRope) y = rope8(y, tab[dv], tab[dmask + 1 + dv]);
    const HeadSlot slot = slots[v >> p.vpd_log2];
    dst[slot.base + s * slot.token_stride + dv] = y;
  }
}

template <int kNorm, bool kScale, bool kRope>
__device__ __noinline__ void process_rows(const NormRopeParams& p, const uint8_t* smem, int stage,
                                          int t, int b, int s0, int count, int lane) {
  const uint4* w = kNorm != 0 ? reinterpret_cast<const uint4*>(smem + p.weight_off[t]) : nullptr;
  const HeadSlot* slots = reinterpret_cast<const HeadSlot*>(smem + p.head_off);
  uint4* dst = p.dst[t] + static_cast<long long>(b) * p.item_vecs;
  const int dmask = (1 << p.vpd_log2) - 1;
  const int nvec = p.heads << p.vpd_log2;
  const int nvec_all = (p.groups * p.hg) << p.vpd_log2;
  for (int r = 0; r < count; ++r) {
    const int s = s0 + r;
    const uint4* row = reinterpret_cast<const uint4*>(smem + p.ring_off + stage * p.stage_bytes +
                                                      r * p.row_bytes);
    const float4* tab = reinterpret_cast<const float4*>(
        smem + p.table_off + stage * p.table_bytes + r * (32 << p.vpd_log2));
    process_row<kNorm, kScale, kRope>(p, row, tab, w, p.post_scale[t], dst, slots, s, lane);
    // zero heads past H (head padding of the last groups)
    for (int v = nvec + lane; v < nvec_all; v += 32) {
      const HeadSlot slot = slots[v >> p.vpd_log2];
      dst[slot.base + s * slot.token_stride + (v & dmask)] = make_uint4(0, 0, 0, 0);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) norm_rope_pack_kernel(
    const __grid_constant__ NormRopeParams p, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  RingControl& ctl = *reinterpret_cast<RingControl*>(smem + p.ctl_off);
  const int S = p.stages;
  const int nslots = p.groups * p.hg;
  // norm weights, rounded to bf16 once (the reference multiplies by
  // scale.astype(bf16)); destination head table
  const int ncols = static_cast<int>(p.cols);
  for (int t = 0; t < p.num_tensors; ++t) {
    if (p.weight_off[t] < 0) continue;
    uint32_t* wdst = reinterpret_cast<uint32_t*>(smem + p.weight_off[t]);
    const float2* wsrc = reinterpret_cast<const float2*>(p.weight[t]);
    for (int i = threadIdx.x; i < ncols / 2; i += kThreads) {
      const float2 w2 = __ldg(wsrc + i);
      wdst[i] = pack2(w2.x, w2.y);
    }
  }
  for (int h = threadIdx.x; h < nslots; h += kThreads)
    reinterpret_cast<HeadSlot*>(smem + p.head_off)[h] = head_slot(p, h);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&ctl.full[i]), 1);
      mbar_init(smem_u32(&ctl.empty[i]), 1);
    }
    ctl.abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort_flag = &ctl.abort_flag;
  const int G = gridDim.x;

  if (threadIdx.x < 32) {
    // ---------------------------------------------------------------- producer
    const int lane = threadIdx.x;
    if (lane >= kProducerLanes) return;
    const uint64_t policy = l2_policy_evict_first();
    int issued = 0;  // this lane's items issued: n = lane + kProducerLanes * k, k < issued
    for (int n = lane;; n += kProducerLanes) {
      const int item = blockIdx.x + n * G;
      if (item >= p.items) break;
      const int stage = n % S;
      const int round = n / S;
      if (round > 0 &&
          !mbar_wait(smem_u32(&ctl.empty[stage]), static_cast<uint32_t>((round - 1) & 1),
                     abort_flag, status, kDevTimeoutLoad))
        break;
      fill_stage(p, smem, item, stage, smem_u32(&ctl.full[stage]), policy);
      ++issued;
    }
    // Before leaving, wait (bounded) until this lane's fills have landed: if
    // the consumers abort, nothing else would keep the CTA alive while copies
    // into its shared memory are in flight. A fill superseded by a later fill
    // of the same stage (item m + S or later) has landed already; its phase
    // parity may have come round again, so it is skipped.
    const int last = issued > 0 ? lane + kProducerLanes * (issued - 1) : -1;
    const int max_last = __reduce_max_sync((1u << kProducerLanes) - 1, last);
    for (int k = issued - 1; k >= 0; --k) {
      const int m = lane + kProducerLanes * k;
      if (m + S <= max_last) break;
      mbar_wait_drain(smem_u32(&ctl.full[m % S]), static_cast<uint32_t>((m / S) & 1), status);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int warp = (threadIdx.x >> 5) - 1;
  const int lane = threadIdx.x & 31;
  for (int n = warp, item = blockIdx.x + warp * G; item < p.items;
       n += kConsumerWarps, item += kConsumerWarps * G) {
    const int stage = n % S;
    if (!mbar_wait(smem_u32(&ctl.full[stage]), static_cast<uint32_t>((n / S) & 1), abort_flag,
                   status, kDevTimeoutSoftmax))
      return;
    int t, b, s0, count;
    item_coords(p, item, t, b, s0, count);
    const int norm = p.weight_off[t] < 0 ? 0 : (p.per_head ? 2 : 1);
    const bool scale = p.post_scale[t] != 1.0f;
    const bool rope = (p.rope_mask >> t) & 1;
    const int mode = norm * 4 + (scale ? 2 : 0) + (rope ? 1 : 0);
    switch (mode) {
#define VX_ROWS(m, N, SC, RO) \
  case m: process_rows<N, SC, RO>(p, smem, stage, t, b, s0, count, lane); break;
      VX_ROWS(0, 0, false, false)
      VX_ROWS(1, 0, false, true)
      VX_ROWS(2, 0, true, false)
      VX_ROWS(3, 0, true, true)
      VX_ROWS(4, 1, false, false)
      VX_ROWS(5, 1, false, true)
      VX_ROWS(6, 1, true, false)
      VX_ROWS(7, 1, true, true)
      VX_ROWS(8, 2, false, false)
      VX_ROWS(9, 2, false, true)
      VX_ROWS(10, 2, true, false)
      VX_ROWS(11, 2, true, true)
#undef VX_ROWS
      default: break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&ctl.empty[stage]));
  }
}

}  // namespace prologue
}  // namespace vx
