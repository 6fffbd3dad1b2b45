// Neighborhood attention with two decoupled query streams per CTA (sm_100a).
//
// Same building blocks as attn_fwd_kernel (tcgen05 MMAs with TMEM
// accumulators, TMA tiles, the NaGeo window geometry and masks, the online
// softmax), different schedule. There, a CTA's two query tiles are two
// adjacent query boxes that walk one key union together: a key tile only one
// box needs leaves the other softmax warpgroup idle, and every unit boundary
// (the next unit's Q load, the epilogue) idles the tensor core. Here each
// softmax warpgroup owns a stream of its own single-box units
//
//   stream t of CTA c: units 2c + t, 2c + t + 2G, 2c + t + 4G, ...   (G = grid)
//
// with its own Q, K and V slots in shared memory (one each, 32 KB at
// head_dim 128: 192 KB in all), and the TMA producer and the MMA issuer poll
// both streams without blocking, issuing whichever stream's next load / MMA
// group is ready. The tensor core interleaves the two streams' MMAs, so one
// stream's softmax, boundary or key-tile loads overlap the other stream's
// MMAs.
//
// Per stream and unit of n key tiles, the MMA groups in issue order are
//   G0 = S(0);  Gj = PV(j-1), S(j)  (1 <= j < n);  Gn = PV(n-1)
// (a PV before the S that overwrites its P columns), and the loads
//   Q + K(0), V(0), K(1), V(1), ..., K(n-1), V(n-1)
// each into its stream's single slot once the MMAs that read the previous
// content completed (K(j+1) after S(j), V(j+1) after PV(j), the next unit's Q
// after this unit's last S). Every wait is bounded as in attn_fwd_kernel; the
// polling loops give up after the same cycle limit without progress.
#pragma once

#include "attn_sm100.cuh"

namespace vx {
namespace na_stream {

using attn::kBlockM;
using attn::kBlockN;
using attn::kHalfBytes;
using attn::kRescaleThreshold;
using attn::kThreads;

enum : int {
  kQFull = 0,     // 2 (per stream): Q landed
  kQEmpty = 2,    // 2: the unit's last S MMA completed (Q free)
  kKFull = 4,     // 2: K(j) landed
  kKEmpty = 6,    // 2: S(j) completed (K slot free)
  kVFull = 8,     // 2: V(j) landed
  kVEmpty = 10,   // 2: PV(j) completed (V slot free)
  kSFull = 12,    // 2: S(j) completed
  kPFull = 14,    // 2: all 128 rows of P(j) written (128 arrivals)
  kOFull = 16,    // 2: the unit's last PV completed
  kOFree = 18,    // 2: the epilogue has read O (128 arrivals)
  kDrain = 20,    // 1
  kNumBars = 21,
};
constexpr uint32_t kTmemSlotOff = 8 * kNumBars;
constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
static_assert(kAbortOff + 4 <= 256, "control block exceeds its reservation");

template <int HD>
struct Layout {
  static constexpr uint32_t kTileBytes = 128u * HD * 2u;
  static constexpr uint32_t kSmemQ = 0;                          // Q_t at kSmemQ + t * tile
  static constexpr uint32_t kSmemK = 2 * kTileBytes;             // K_t
  static constexpr uint32_t kSmemV = 4 * kTileBytes;             // V_t
  static constexpr uint32_t kSmemBar = 6 * kTileBytes;
  static constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;  // + control block + alignment
  static constexpr uint32_t kTmemO = 256;                        // O_t at kTmemO + HD * t
};

// Stream t's k-th unit, or -1 when the stream is done.
__device__ __forceinline__ int stream_unit(int t, int k, int num_units) {
  const long long u = 2LL * blockIdx.x + t + 2LL * k * gridDim.x;
  return u < num_units ? static_cast<int>(u) : -1;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    na_stream_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ attn::NaParams p) {
  using Geo = attn::NaGeo<2, 4, 16, HD>;
  using Ly = Layout<HD>;
  constexpr uint32_t kTileBytes = Ly::kTileBytes;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + Ly::kSmemBar + 8u * i; };
  volatile uint32_t* tmem_slot =
      reinterpret_cast<volatile uint32_t*>(smem + Ly::kSmemBar + kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Ly::kSmemBar + kAbortOff);
  int* status = p.status;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kQFull + t), 1);
      mbar_init(bar(kQEmpty + t), 1);
      mbar_init(bar(kKFull + t), 1);
      mbar_init(bar(kKEmpty + t), 1);
      mbar_init(bar(kVFull + t), 1);
      mbar_init(bar(kVEmpty + t), 1);
      mbar_init(bar(kSFull + t), 1);
      mbar_init(bar(kPFull + t), 128);
      mbar_init(bar(kOFull + t), 1);
      mbar_init(bar(kOFree + t), 128);
    }
    mbar_init(bar(kDrain), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(sbase + Ly::kSmemBar + kTmemSlotOff, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // A polling loop that made no progress for this long gives up (as a
  // bounded mbarrier wait would).
  auto stalled = [&](long long& t_idle, bool progressed, int code) -> bool {
    if (progressed) {
      t_idle = clock64();
      return false;
    }
    if (*abort_flag) return true;
    if (clock64() - t_idle > kWaitLimitCycles) {
      *abort_flag = 1;
      atomicOr(status, code);
      return true;
    }
    return false;
  };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      int k_unit[2] = {0, 0};    // units started per stream
      int unit[2], n[2], item[2];  // current unit, its key tiles, next load (0 = Q + K(0))
      int q_loads[2] = {0, 0}, k_loads[2] = {0, 0}, v_loads[2] = {0, 0};
      bool done[2];
      for (int t = 0; t < 2; ++t) {
        unit[t] = stream_unit(t, 0, p.num_units);
        done[t] = unit[t] < 0;
        n[t] = done[t] ? 0 : Geo(p, unit[t]).num_kv_tiles();
        item[t] = 0;
      }
      long long t_idle = clock64();
      bool aborted = false;
      while (!(done[0] && done[1])) {
        bool progressed = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (done[t]) continue;
          Geo geo(p, unit[t]);
          const int it = item[t];
          if (it == 0) {  // Q and K(0) of a new unit
            if (!mbar_try_wait(bar(kQEmpty + t), (q_loads[t] & 1) ^ 1) ||
                !mbar_try_wait(bar(kKEmpty + t), (k_loads[t] & 1) ^ 1))
              continue;
            mbar_expect_tx(bar(kQFull + t), kTileBytes);
            geo.load_q(&tm_q, 0, sbase + Ly::kSmemQ + t * kTileBytes, bar(kQFull + t), pol_q);
            mbar_expect_tx(bar(kKFull + t), kTileBytes);
            geo.load_kv(&tm_k, 0, sbase + Ly::kSmemK + t * kTileBytes, bar(kKFull + t), pol_kv);
            ++q_loads[t];
            ++k_loads[t];
          } else if (it & 1) {  // V(j), j = (it - 1) / 2
            if (!mbar_try_wait(bar(kVEmpty + t), (v_loads[t] & 1) ^ 1)) continue;
            mbar_expect_tx(bar(kVFull + t), kTileBytes);
            geo.load_kv(&tm_v, (it - 1) >> 1, sbase + Ly::kSmemV + t * kTileBytes,
                        bar(kVFull + t), pol_kv);
            ++v_loads[t];
          } else {  // K(j), j = it / 2
            if (!mbar_try_wait(bar(kKEmpty + t), (k_loads[t] & 1) ^ 1)) continue;
            mbar_expect_tx(bar(kKFull + t), kTileBytes);
            geo.load_kv(&tm_k, it >> 1, sbase + Ly::kSmemK + t * kTileBytes, bar(kKFull + t),
                        pol_kv);
            ++k_loads[t];
          }
          progressed = true;
          if (++item[t] == 2 * n[t]) {  // items 0 .. 2n-1: Q+K0, V0, K1, V1, ..., V(n-1)
            unit[t] = stream_unit(t, ++k_unit[t], p.num_units);
            done[t] = unit[t] < 0;
            n[t] = done[t] ? 0 : Geo(p, unit[t]).num_kv_tiles();
            item[t] = 0;
          }
        }
        if (stalled(t_idle, progressed, kDevTimeoutLoad)) {
          aborted = true;
          break;
        }
      }
      if (aborted || *abort_flag) {
        // Drain: the last load into each slot must land before the CTA exits.
        for (int t = 0; t < 2; ++t) {
          if (q_loads[t] > 0) mbar_wait_drain(bar(kQFull + t), (q_loads[t] - 1) & 1, status);
          if (k_loads[t] > 0) mbar_wait_drain(bar(kKFull + t), (k_loads[t] - 1) & 1, status);
          if (v_loads[t] > 0) mbar_wait_drain(bar(kVFull + t), (v_loads[t] - 1) & 1, status);
        }
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int k_unit[2] = {0, 0}, unit[2], n[2], grp[2];
      int q_uses[2] = {0, 0}, k_uses[2] = {0, 0}, v_uses[2] = {0, 0};
      int p_count[2] = {0, 0}, o_units[2] = {0, 0};
      bool done[2];
      uint64_t q_desc[2], k_desc[2], v_desc[2];
      for (int t = 0; t < 2; ++t) {
        unit[t] = stream_unit(t, 0, p.num_units);
        done[t] = unit[t] < 0;
        n[t] = done[t] ? 0 : Geo(p, unit[t]).num_kv_tiles();
        grp[t] = 0;
        q_desc[t] = sdesc_sw128(sbase + Ly::kSmemQ + t * kTileBytes, 16, 1024);
        k_desc[t] = sdesc_sw128(sbase + Ly::kSmemK + t * kTileBytes, 16, 1024);
        v_desc[t] = sdesc_sw128(sbase + Ly::kSmemV + t * kTileBytes, kHalfBytes, 1024);
      }
      long long t_idle = clock64();
      while (!(done[0] && done[1])) {
        bool progressed = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (done[t]) continue;
          const int g = grp[t], nt = n[t];
          const bool has_pv = g > 0;   // PV(g - 1)
          const bool has_s = g < nt;   // S(g)
          // readiness (parity tests only; nothing is consumed by a test)
          if (g == 0 && !mbar_try_wait(bar(kQFull + t), q_uses[t] & 1)) continue;
          if (has_s && !mbar_try_wait(bar(kKFull + t), k_uses[t] & 1)) continue;
          if (has_pv) {
            if (g == 1 && !mbar_try_wait(bar(kOFree + t), (o_units[t] & 1) ^ 1)) continue;
            if (!mbar_try_wait(bar(kPFull + t), p_count[t] & 1)) continue;
            if (!mbar_try_wait(bar(kVFull + t), v_uses[t] & 1)) continue;
          }
          tc_fence_after();
          if (has_pv) {
            attn::issue_pv_half<HD>(tmem + Ly::kTmemO + HD * t, tmem + 128 * t, v_desc[t], 0, g > 1);
            attn::issue_pv_half<HD>(tmem + Ly::kTmemO + HD * t, tmem + 128 * t, v_desc[t], 1, true);
            tc_commit(bar(kVEmpty + t));
            ++v_uses[t];
            ++p_count[t];
            if (g == nt) {
              tc_commit(bar(kOFull + t));
              ++o_units[t];
            }
          }
          if (has_s) {
            attn::issue_qk<HD>(tmem + 128 * t, q_desc[t], k_desc[t]);
            tc_commit(bar(kSFull + t));
            tc_commit(bar(kKEmpty + t));
            ++k_uses[t];
            if (g == 0) ++q_uses[t];
            if (g == nt - 1) tc_commit(bar(kQEmpty + t));  // the unit's last S read Q
          }
          progressed = true;
          if (++grp[t] > nt) {
            unit[t] = stream_unit(t, ++k_unit[t], p.num_units);
            done[t] = unit[t] < 0;
            n[t] = done[t] ? 0 : Geo(p, unit[t]).num_kv_tiles();
            grp[t] = 0;
          }
        }
        if (stalled(t_idle, progressed, kDevTimeoutMma)) break;
      }
      // Drain: no MMA may still be running when TMEM is released.
      tc_commit(bar(kDrain));
      mbar_wait_drain(bar(kDrain), 0, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;     // stream
    const int quad = warp & 3;   // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + lane_off;
    const uint32_t t_o = tmem + Ly::kTmemO + t * HD + lane_off;
    const float scale_log2 = p.scale_log2;
    int s_count = 0, o_units = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int u = stream_unit(t, k, p.num_units);
      if (u < 0) break;
      Geo geo(p, u);
      const int n_kv = geo.num_kv_tiles();
      geo.softmax_setup(0, row);
      float m_used = attn::neg_inf();
      float l_sum = 0.f;
      for (int j = 0; j < n_kv; ++j) {
        uint32_t cm[4];
        const uint32_t active = geo.chunk_masks(j, cm);
        ok = mbar_wait(bar(kSFull + t), s_count & 1, abort_flag, status, kDevTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, sr[c]);
        tmem_wait_ld_only();
#pragma unroll
        for (int c = 0; c < 4; ++c) attn::pin32(sr[c]);
        geo.apply_masks(cm, active, sr);
        float mx0 = attn::neg_inf(), mx1 = attn::neg_inf(), mx2 = attn::neg_inf(),
              mx3 = attn::neg_inf();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (!((active >> c) & 1u)) continue;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            mx0 = fmax3(mx0, __uint_as_float(sr[c][i + 0]), __uint_as_float(sr[c][i + 1]));
            mx1 = fmax3(mx1, __uint_as_float(sr[c][i + 2]), __uint_as_float(sr[c][i + 3]));
            mx2 = fmax3(mx2, __uint_as_float(sr[c][i + 4]), __uint_as_float(sr[c][i + 5]));
            mx3 = fmax3(mx3, __uint_as_float(sr[c][i + 6]), __uint_as_float(sr[c][i + 7]));
          }
        }
        const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale_log2;
        const float m_new = fmaxf(m_used, mx);
        const bool need = m_new > m_used + kRescaleThreshold;
        float alpha = 1.f;
        if (need) alpha = ex2_approx(m_used - m_new);
        const bool rescale_o = j > 0 && __any_sync(0xffffffffu, need);
        if (need) {
          l_sum *= alpha;
          m_used = m_new;
        }
        const float neg_m = (m_used == attn::neg_inf()) ? 0.f : -m_used;
        uint64_t ls2 = f2_pack(0.f, 0.f);
        const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(neg_m, neg_m);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
          if (!((active >> c) & 1u)) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = 0u;
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c][2 * i]),
                                       __uint_as_float(sr[c][2 * i + 1])),
                               sc2, nm2),
                        x0, x1);
              const float e0 = ex2_approx(x0);
              const float e1 = ex2_approx(x1);
              ls2 = f2_add(ls2, f2_pack(e0, e1));
              pk[i] = pack_bf16x2(e0, e1);
            }
          }
          tmem_st16(t_s + c * 16, pk);
        }
        if (rescale_o) {
          // O holds PV(0 .. j-1): S(j) was issued after PV(j-1), and its
          // commit tracks every earlier MMA of this issuer.
#pragma unroll 1
          for (int cc = 0; cc < HD / 32; ++cc) {
            uint32_t orr[32];
            tmem_ld32(t_o + cc * 32, orr);
            tmem_wait_ld(orr);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
            tmem_st32(t_o + cc * 32, orr);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(kPFull + t));
        float ls0, ls1;
        f2_unpack(ls2, ls0, ls1);
        l_sum += ls0 + ls1;
        ++s_count;
      }
      if (!ok) break;
      ok = mbar_wait(bar(kOFull + t), o_units & 1, abort_flag, status, kDevTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float inv_l = l_sum > 0.f ? 1.f / l_sum : 0.f;
      uint32_t pk[HD / 32][16];
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t orr[32];
        tmem_ld32(t_o + c * 32, orr);
        tmem_wait_ld(orr);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[c][i] = pack_bf16x2(__uint_as_float(orr[2 * i]) * inv_l,
                                 __uint_as_float(orr[2 * i + 1]) * inv_l);
      }
      tc_fence_before();
      mbar_arrive(bar(kOFree + t));  // the stream's next unit may overwrite O
      ++o_units;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) geo.store_row_chunk(0, row, c, pk[c]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace na_stream
}  // namespace vx
