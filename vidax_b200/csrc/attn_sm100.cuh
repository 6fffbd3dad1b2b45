// Warp-specialised tcgen05/TMEM attention forward for sm_100a (head_dim 128,
// bf16 in/out, fp32 softmax and accumulation).
//
// One CTA owns a pair of 128-row query tiles (Q0, Q1) of one (batch, head)
// and streams 128-key K/V tiles through a two-stage TMA ring:
//
//   warps 0-3  softmax warpgroup for Q0   (thread i owns query row i)
//   warps 4-7  softmax warpgroup for Q1
//   warp  8    TMA producer (one elected lane)
//   warp  9    TMEM allocator + MMA issuer (one elected lane)
//
// Tensor memory (512 columns x 128 lanes, fp32):
//   [  0,128) S0 = Q0 K^T   (P0 = softmax numerators, bf16, aliases cols [0,64))
//   [128,256) S1 = Q1 K^T   (P1 aliases cols [128,192))
//   [256,384) O0 += P0 V
//   [384,512) O1 += P1 V
//
// MMA order per KV tile j (ping-pong so the tensor core works on one query
// tile while the other one's softmax runs):
//   PV0(j) ; S0(j+1) ; PV1(j) ; S1(j+1)
// S0(j+1) overwrites the columns PV0(j) reads P0 from; tcgen05.mma ops issued
// by one thread execute in issue order, which orders that reuse.
//
// Online softmax uses a lazy rescale: the running row maximum used in the
// exponent only moves when the new maximum exceeds it by more than
// kRescaleThreshold (log2 units), so the O accumulator in TMEM is rescaled
// rarely; P values stay <= 2^kRescaleThreshold, well inside bf16 range. The
// final O / l is exact regardless of which maximum was used.
//
// The geometry policy (`Geo`) decides which rows form the query tiles, which
// K/V tiles are visited, how keys are masked and where output rows go: the
// dense policy serves full attention, the neighborhood policy serves 3-D
// windowed attention with the same pipeline.
#pragma once

#include "sm100_common.cuh"

namespace vx {
namespace attn {

constexpr int kBlockM = 128;  // query rows per tile (one softmax warpgroup)
constexpr int kBlockN = 128;  // keys per K/V tile
constexpr int kStages = 2;
constexpr int kThreads = 320;
constexpr uint32_t kHalfBytes = 128u * 64u * 2u;  // 128 rows x 64 cols: one 128B-swizzle slab
constexpr float kRescaleThreshold = 8.0f;

// Head-dimension dependent sizes (head_dim 64 or 128). A 128-row tile of
// head_dim D is D/64 swizzle slabs of kHalfBytes. A K / V stage holds KVT
// tiles: one shared by both query tiles, or one per query tile when the two
// query tiles belong to different heads (Geo::kKVTiles = 2).
template <int HD, int KVT = 1>
struct Dims {
  static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
  static_assert(KVT == 1 || KVT == 2, "one or two K / V tiles per stage");
  static constexpr int kHeadDim = HD;
  static constexpr int kHalves = HD / 64;
  static constexpr uint32_t kTileBytes = 128u * HD * 2u;
  static constexpr uint32_t kKVStageBytes = KVT * kTileBytes;
  static constexpr uint32_t kSmemQ = 0;
  static constexpr uint32_t kSmemK = kSmemQ + 2 * kTileBytes;
  static constexpr uint32_t kSmemV = kSmemK + kStages * kKVStageBytes;
  static constexpr uint32_t kSmemBar = kSmemV + kStages * kKVStageBytes;
  static constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;  // + control block + alignment
  static constexpr uint32_t kTmemO = 256;                        // O_t at kTmemO + HD * t
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory per CTA");
};
// dynamic shared memory of attn_fwd_kernel<Geo, ...>
template <class Geo>
constexpr uint32_t smem_bytes() {
  return Dims<Geo::kHeadDim, Geo::kKVTiles>::kSmemBytes;
}

// barrier slots
enum : int {
  kQFull = 0,      // 2: [0] = Q0 + the unit's first K, [1] = Q1
  kQEmpty = 2,     // 1: the unit's MMAs are done with Q
  kKVFull = 3,     // kStages: V(j) + K(j+1) landed (stage = global tile % kStages)
  kKEmpty = 5,     // kStages
  kVEmpty = 7,     // kStages
  kSFull = 9,      // 2
  kPFull = 11,     // 2: all P columns of query tile t written
  kOFull = 13,     // 2: the unit's last PV of query tile t completed
  kOFree = 15,     // 2: the epilogue has read O_t
  kDrain = 17,     // 1
  kUnitFull = 18,  // 2: unit ring slot written by the scheduler
  kUnitEmpty = 20, // 2: unit ring slot read by the MMA issuer and all softmax threads
  kClc = 22,       // 1: cluster-launch-control response landed
  kNumBars = 23,
};
// control block (offsets from the barrier base, which is 1024-aligned)
constexpr uint32_t kTmemSlotOff = 8 * kNumBars;
constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
constexpr uint32_t kUnitRingOff = kAbortOff + 4;                   // 2 ints
constexpr uint32_t kClcRespOff = (kUnitRingOff + 8 + 15) & ~15u;   // 16 bytes, 16-aligned
static_assert(kClcRespOff + 16 <= 256, "control block exceeds its reservation");
constexpr int kUnitConsumers = 1 + 256;  // MMA issuer + every softmax thread

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, false, false);  // Q K^T: both K-major
template <int HD>
__host__ __device__ constexpr uint32_t idesc_pv() {  // P V: V is N-major
  return idesc_bf16_f32(128, HD, false, true);
}

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// S_t = Q_t K^T over head_dim 128 (8 MMAs of K=16). Each operand tile is two
// 128B-swizzled halves of 64 columns; within a half the K step advances the
// descriptor start address by 32 bytes. `q_desc` / `k_desc` are the tiles'
// base descriptors; the per-step offsets are compile-time constants added to
// the start-address field (in 16-byte units, no carry out of the field since
// shared memory is below 256 KB).
template <int HD>
__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint64_t q_desc, uint64_t k_desc) {
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4);
    mma_ss(tmem_s, q_desc + off, k_desc + off, kIdescS, kk > 0 ? 1u : 0u);
  }
}

// O_t (+)= P_t V with P_t read from tensor memory (8 columns per K=16 step)
// and V an N-major 128B-swizzled tile (`v_desc`): 16 keys per step = 2048
// bytes; the two 64-column halves of head_dim are kHalfBytes apart (leading
// byte offset). `half` selects keys [0, 64) or [64, 128) of the tile (4 MMAs
// each).
template <int HD>
__device__ __forceinline__ void issue_pv_half(uint32_t tmem_o, uint32_t tmem_p, uint64_t v_desc,
                                              int half, bool accumulate) {
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    const int kk = half * 4 + k4;
    mma_ts(tmem_o, tmem_p + kk * 8, v_desc + static_cast<uint64_t>((kk * 2048) >> 4),
           idesc_pv<HD>(), (accumulate || kk > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ void pin32(uint32_t (&r)[32]) { asm volatile("" : VX_RW32(r)); }

// Work scheduling of attn_fwd_kernel (template parameter kSched).
enum : int {
  kSchedSingle = 0,  // grid = units, each CTA runs exactly its own unit
  kSchedStride = 1,  // grid = min(units, SMs), CTA b runs units b, b + grid, ...
  kSchedSteal = 2,   // grid = units, running CTAs take over unlaunched ones (CLC)
};

template <class Geo, int kSched>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ typename Geo::Params p) {
  using Dm = Dims<Geo::kHeadDim, Geo::kKVTiles>;
  constexpr int HD = Geo::kHeadDim;
  constexpr uint32_t kTileBytes = Dm::kTileBytes;
  constexpr uint32_t kKVStage = Dm::kKVStageBytes;
  constexpr uint32_t kSmemQ = Dm::kSmemQ, kSmemK = Dm::kSmemK, kSmemV = Dm::kSmemV;
  constexpr uint32_t kSmemBar = Dm::kSmemBar;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + kSmemBar + 8u * i; };
  volatile uint32_t* tmem_slot =
      reinterpret_cast<volatile uint32_t*>(smem + kSmemBar + kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemBar + kAbortOff);
  int* status = p.status;
  volatile int* unit_ring = reinterpret_cast<volatile int*>(smem + kSmemBar + kUnitRingOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar(kQFull + 0), 1);
    mbar_init(bar(kQFull + 1), 1);
    mbar_init(bar(kQEmpty), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kKVFull + s), 1);
      mbar_init(bar(kKEmpty + s), 1);
      mbar_init(bar(kVEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kSFull + t), 1);
      mbar_init(bar(kPFull + t), 128);
      mbar_init(bar(kOFull + t), 1);
      mbar_init(bar(kOFree + t), 128);
    }
    mbar_init(bar(kDrain), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(kUnitFull + i), 1);
      mbar_init(bar(kUnitEmpty + i), kUnitConsumers);
    }
    mbar_init(bar(kClc), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(sbase + kSmemBar + kTmemSlotOff, 512);
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

  // Schedule: each CTA processes its own unit (blockIdx.x) first. Then, with
  // kSchedStride, units blockIdx.x + gridDim.x, ...; with kSchedSteal it asks
  // the hardware (cluster launch control) to cancel a CTA that has not
  // launched yet and processes that CTA's unit instead, until none is left --
  // a persistent, dynamically balanced schedule that adapts when other
  // kernels (e.g. NCCL's) hold some SMs. The producer thread is the
  // scheduler: it publishes the unit sequence (ending with -1) through a
  // two-slot ring in shared memory that the MMA issuer and the softmax
  // threads read. Barrier phases run on across units: KV tiles
  // are numbered globally (g) for the ring, and each role counts the units
  // it has taken part in.
  auto next_unit = [&](int k, int code, int& u) -> bool {
    // consumer side of the unit ring: k-th published unit
    if (!mbar_wait(bar(kUnitFull + (k & 1)), (k >> 1) & 1, abort_flag, status, code)) return false;
    u = unit_ring[k & 1];
    mbar_arrive(bar(kUnitEmpty + (k & 1)));
    return true;
  };
  if (warp == 8) {
    // ------------------------------------------------------------ producer
    // Per unit: (after the previous unit's MMAs released Q) Q0 + first K on
    // Q_FULL[0], Q1 on Q_FULL[1]; then per KV tile j the pair V(j), K(j+1) on
    // one KV_FULL barrier, so the MMA issuer waits once per tile.
    if (lane == 0) {
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      const uint32_t clc_resp = sbase + kSmemBar + kClcRespOff;
      uint32_t g = 0;   // global index of the unit's first KV tile
      int qi = 0;       // units with work issued
      int last_pair = -1;
      int clc_issued = 0, clc_done = 0;
      bool ok = true;
      auto publish = [&](int k, int u) -> bool {
        if (!mbar_wait(bar(kUnitEmpty + (k & 1)), ((k >> 1) & 1) ^ 1, abort_flag, status,
                       kDevTimeoutLoad))
          return false;
        unit_ring[k & 1] = u;
        mbar_arrive(bar(kUnitFull + (k & 1)));
        return true;
      };
      int u = blockIdx.x;
      ok = publish(0, u);
      for (int k = 1; ok && u >= 0; ++k) {
        Geo geo(p, u);
        const int n = geo.num_kv_tiles();
        if (kSched == kSchedSteal) {
          // request the next unit now; the answer is needed only after this
          // unit's loads are issued
          mbar_expect_tx(bar(kClc), 16);
          clc_try_cancel(clc_resp, bar(kClc));
          ++clc_issued;
        }
        if (n > 0) {
          const int sk = g % kStages;
          ok = mbar_wait(bar(kQEmpty), (qi & 1) ^ 1, abort_flag, status, kDevTimeoutLoad) &&
               mbar_wait(bar(kKEmpty + sk), ((g / kStages) & 1) ^ 1, abort_flag, status,
                         kDevTimeoutLoad);
          if (!ok) break;
          mbar_expect_tx(bar(kQFull + 0), kTileBytes + kKVStage);
          geo.load_q(&tm_q, 0, sbase + kSmemQ, bar(kQFull + 0), pol_q);
          geo.load_kv(&tm_k, 0, sbase + kSmemK + sk * kKVStage, bar(kQFull + 0), pol_kv);
          mbar_expect_tx(bar(kQFull + 1), kTileBytes);
          geo.load_q(&tm_q, 1, sbase + kSmemQ + kTileBytes, bar(kQFull + 1), pol_q);
          for (int j = 0; j < n; ++j) {
            const uint32_t gj = g + j;
            const int s = gj % kStages;
            const uint32_t ph = (gj / kStages) & 1;
            const bool has_next = j + 1 < n;
            const int s1 = (gj + 1) % kStages;
            const uint32_t ph1 = ((gj + 1) / kStages) & 1;
            if (!mbar_wait(bar(kVEmpty + s), ph ^ 1, abort_flag, status, kDevTimeoutLoad)) {
              ok = false;
              break;
            }
            if (has_next &&
                !mbar_wait(bar(kKEmpty + s1), ph1 ^ 1, abort_flag, status, kDevTimeoutLoad)) {
              ok = false;
              break;
            }
            mbar_expect_tx(bar(kKVFull + s), has_next ? 2 * kKVStage : kKVStage);
            geo.load_kv(&tm_v, j, sbase + kSmemV + s * kKVStage, bar(kKVFull + s), pol_kv);
            if (has_next)
              geo.load_kv(&tm_k, j + 1, sbase + kSmemK + s1 * kKVStage, bar(kKVFull + s),
                          pol_kv);
            last_pair = static_cast<int>(gj);
          }
          if (!ok) break;
          g += n;
          ++qi;
        }
        int nu = -1;
        if (kSched == kSchedStride && u + static_cast<int>(gridDim.x) < p.num_units)
          nu = u + static_cast<int>(gridDim.x);
        if (kSched == kSchedSteal) {
          if (!mbar_wait(bar(kClc), clc_done & 1, abort_flag, status, kDevTimeoutLoad)) break;
          ++clc_done;
          int x;
          if (clc_query(clc_resp, x)) nu = x;
          fence_proxy_async_smem();  // the read precedes the next async response write
        }
        ok = publish(k, nu);
        u = nu;
      }
      if (*abort_flag) {
        // Drain: wait for the most recent loads into each stage and into Q
        // to land so no TMA write targets this CTA's shared memory after it
        // exits. Only the last load per stage can be pending.
        for (int gj = last_pair; gj >= 0 && gj > last_pair - kStages; --gj)
          mbar_wait_drain(bar(kKVFull + gj % kStages), (gj / kStages) & 1, status);
        if (qi > 0) {
          mbar_wait_drain(bar(kQFull + 0), (qi - 1) & 1, status);
          mbar_wait_drain(bar(kQFull + 1), (qi - 1) & 1, status);
        }
        if (clc_issued > clc_done) mbar_wait_drain(bar(kClc), clc_done & 1, status);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // Per unit and KV tile j: release K(j) (its S MMAs were issued earlier),
    // wait for V(j) + K(j+1), then for each query tile t that needs j:
    //   PV_t(j) once P_t(j) is published (and, for the unit's first PV, once
    //   the previous unit's epilogue has read O_t), then S_t(j+1).
    // A query tile that does not need a KV tile skips it (neighborhood
    // geometry; the dense one needs every tile).
    if (lane == 0) {
      const uint64_t q_desc[2] = {sdesc_sw128(sbase + kSmemQ, 16, 1024),
                                  sdesc_sw128(sbase + kSmemQ + kTileBytes, 16, 1024)};
      static_assert(kStages == 2, "descriptor selection below assumes two stages");
      const uint64_t k_desc0 = sdesc_sw128(sbase + kSmemK, 16, 1024);
      const uint64_t v_desc0 = sdesc_sw128(sbase + kSmemV, kHalfBytes, 1024);
      // stage 1 = stage 0 + kKVStage in the start-address field; with a K / V
      // tile per query tile, query tile t's tile is t * kTileBytes further
      constexpr uint64_t kStageStep = kKVStage >> 4;
      auto kv_tile = [](int t) -> uint64_t {
        return Geo::kKVTiles == 2 ? static_cast<uint64_t>(t) * (kTileBytes >> 4) : 0ull;
      };
      uint32_t g = 0;
      int qi = 0;
      int p_count[2] = {0, 0};  // P publications consumed per query tile
      int o_units[2] = {0, 0};  // units in which query tile t accumulated O
      bool ok = true;
      for (int k = 0; ok; ++k) {
        int u;
        if (!next_unit(k, kDevTimeoutMma, u) || u < 0) break;
        Geo geo(p, u);
        const int n = geo.num_kv_tiles();
        if (n == 0) continue;
        // last tiles first: the scan over the key union runs while Q loads
        const int last[2] = {geo.last_tile(0), geo.last_tile(1)};
        ok = mbar_wait(bar(kQFull + 0), qi & 1, abort_flag, status, kDevTimeoutMma) &&
             mbar_wait(bar(kQFull + 1), qi & 1, abort_flag, status, kDevTimeoutMma);
        if (!ok) break;
        bool first_pv[2] = {true, true};
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (geo.needs(t, 0)) {
            issue_qk<HD>(tmem + 128 * t, q_desc[t],
                         k_desc0 + ((g % kStages) ? kStageStep : 0) + kv_tile(t));
            tc_commit(bar(kSFull + t));
          }
        }
        // Q is released as soon as the unit's last S MMA has been issued, so
        // the next unit's Q loads while this unit's last PVs and epilogue run.
        bool q_released = false;
        if (n == 1) {
          tc_commit(bar(kQEmpty));
          q_released = true;
        }
        for (int j = 0; ok && j < n; ++j) {
          const uint32_t gj = g + j;
          const int s = gj % kStages;
          const uint32_t ph = (gj / kStages) & 1;
          const int s1 = (gj + 1) % kStages;
          const bool has_next = j + 1 < n;
          const uint64_t v_d = v_desc0 + (s ? kStageStep : 0);
          const uint64_t k_next = k_desc0 + (s1 ? kStageStep : 0);
          tc_commit(bar(kKEmpty + s));  // every S MMA reading K(j) was issued before
          if (!mbar_wait(bar(kKVFull + s), ph, abort_flag, status, kDevTimeoutMma)) break;
          tc_fence_after();
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (geo.needs(t, j)) {
              if (first_pv[t] && !mbar_wait(bar(kOFree + t), (o_units[t] & 1) ^ 1, abort_flag,
                                            status, kDevTimeoutMma)) {
                ok = false;
                break;
              }
              if (!mbar_wait(bar(kPFull + t), p_count[t] & 1, abort_flag, status,
                             kDevTimeoutMma)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_pv_half<HD>(tmem + Dm::kTmemO + HD * t, tmem + 128 * t, v_d + kv_tile(t), 0,
                                !first_pv[t]);
              issue_pv_half<HD>(tmem + Dm::kTmemO + HD * t, tmem + 128 * t, v_d + kv_tile(t), 1,
                                true);
              first_pv[t] = false;
              ++p_count[t];
              if (j == last[t]) tc_commit(bar(kOFull + t));
            }
            if (has_next && geo.needs(t, j + 1)) {
              issue_qk<HD>(tmem + 128 * t, q_desc[t], k_next + kv_tile(t));
              tc_commit(bar(kSFull + t));
            }
          }
          if (!ok) break;
          if (!q_released && j + 2 == n) {  // S(n-1), the unit's last S, was just issued
            tc_commit(bar(kQEmpty));
            q_released = true;
          }
          tc_commit(bar(kVEmpty + s));
        }
        if (!ok) break;
        for (int t = 0; t < 2; ++t)
          if (!first_pv[t]) ++o_units[t];
        g += n;
        ++qi;
      }
      // Drain: no MMA may still be running when TMEM is released.
      tc_commit(bar(kDrain));
      mbar_wait_drain(bar(kDrain), 0, status);
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax
    const int wg = warp >> 2;    // which query tile
    const int quad = warp & 3;   // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_s = tmem + wg * 128 + lane_off;
    const uint32_t t_o = tmem + Dm::kTmemO + wg * HD + lane_off;
    const float scale_log2 = p.scale_log2;
    int s_count = 0;  // S tiles consumed by this query tile (all units)
    int o_units = 0;  // units in which this query tile accumulated O
    bool ok = true;
    for (int k = 0; ok; ++k) {
      int u;
      ok = next_unit(k, kDevTimeoutSoftmax, u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || u < 0) break;
      Geo geo(p, u);
      const int n_kv = geo.num_kv_tiles();
      geo.softmax_setup(wg, row);
      float m_used = neg_inf();
      float l_sum = 0.f;
      int count = 0;  // KV tiles this query tile processed in this unit
      for (int j = 0; j < n_kv; ++j) {
        if (!geo.needs_own(j)) continue;
        // the tile's key masks need no scores: built while S(j) is computed
        uint32_t cm[4];
        const uint32_t active = geo.chunk_masks(j, cm);
        ok = mbar_wait(bar(kSFull + wg), s_count & 1, abort_flag, status, kDevTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, sr[c]);
        tmem_wait_ld_only();
#pragma unroll
        for (int c = 0; c < 4; ++c) pin32(sr[c]);

        geo.apply_masks(cm, active, sr);

        // row max: 3-input max over 128 scores, 4 independent chains
        float mx0 = neg_inf(), mx1 = neg_inf(), mx2 = neg_inf(), mx3 = neg_inf();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (!((active >> c) & 1u)) continue;  // warp-uniform: no visible key
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
        if (need) alpha = ex2_approx(m_used - m_new);  // 0 when m_used = -inf
        // O is rescaled after P is computed (fewer live registers) and before P
        // is published: PV(j) must accumulate into the rescaled O.
        const bool rescale_o = count > 0 && __any_sync(0xffffffffu, need);
        if (need) {
          l_sum *= alpha;
          m_used = m_new;
        }
        const float neg_m = (m_used == neg_inf()) ? 0.f : -m_used;
        // p = 2^(s * scale_log2 - m) on MUFU, packed to bf16 over S's columns.
        // Even columns sum into ls0, odd into ls1. Geometries whose softmax is
        // issue-bound (the neighborhood one, with its masks) do the scaling
        // and the sums two columns per instruction (f32x2); the results are
        // bit-identical (same roundings, same summation order).
        float ls0 = 0.f, ls1 = 0.f;
        uint64_t ls2 = f2_pack(0.f, 0.f);
        const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(neg_m, neg_m);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
          if (!((active >> c) & 1u)) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = 0u;
          } else if (Geo::kPackedSoftmax) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])),
                               sc2, nm2), x0, x1);
              const float e0 = ex2_approx(x0);
              const float e1 = ex2_approx(x1);
              ls2 = f2_add(ls2, f2_pack(e0, e1));
              pk[i] = pack_bf16x2(e0, e1);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float e0 = ex2_approx(fmaf(__uint_as_float(sr[c][2 * i]), scale_log2, neg_m));
              const float e1 =
                  ex2_approx(fmaf(__uint_as_float(sr[c][2 * i + 1]), scale_log2, neg_m));
              ls0 += e0;
              ls1 += e1;
              pk[i] = pack_bf16x2(e0, e1);
            }
          }
          tmem_st16(t_s + c * 16, pk);
        }
        if (Geo::kPackedSoftmax) f2_unpack(ls2, ls0, ls1);
        if (rescale_o) {
          // O is complete up to this query tile's previous KV tile: S(j) was
          // issued after that PV and its commit tracks every earlier MMA.
          // Rescale this warp's 32 rows of O.
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
        mbar_arrive(bar(kPFull + wg));
        l_sum += ls0 + ls1;
        ++s_count;
        ++count;
      }
      if (!ok) break;
      if (count == 0) {
        geo.store_zero_row(wg, row);
        continue;
      }
      ok = mbar_wait(bar(kOFull + wg), o_units & 1, abort_flag, status, kDevTimeoutSoftmax);
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
      // O_t has been read: the next unit's first PV may overwrite it.
      tc_fence_before();
      mbar_arrive(bar(kOFree + wg));
      ++o_units;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) geo.store_row_chunk(wg, row, c, pk[c]);
      // natural-log LSE of the row's scaled logits
      const float lse = l_sum > 0.f ? (m_used + __log2f(l_sum)) * 0.69314718055994531f
                                    : neg_inf();
      geo.store_lse(wg, row, lse);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------------------------------
// Dense geometry: query tiles are consecutive rows of one (batch, head); the
// K/V tiles sweep all valid keys; keys at index >= kv_valid are masked.
// Tensors are BSHD; the tensor maps are 4-D {D, H, S, B}.
struct DenseParams {
  __nv_bfloat16* o;
  long long o_sb, o_ss, o_sh;  // output strides in elements (d stride is 1)
  float* lse;                  // optional (B, H, Sq) fp32
  const int* kv_len;           // optional [B]
  int* status;
  int B, Sq, Sk, H, Hkv;
  int num_qblocks;             // ceil(Sq / 256)
  int num_units;               // num_qblocks * H * B
  float scale_log2;
};

template <int HD>
struct DenseGeo {
  static constexpr int kHeadDim = HD;
  static constexpr bool kPackedSoftmax = false;  // MUFU-bound: scalar arithmetic is as fast
  static constexpr int kKVTiles = 1;             // both query tiles read the same K / V
  using Params = DenseParams;
  const DenseParams& p;
  int b, h, hk, q0, kv_valid;
  int row_global;

  // Work unit u = (query block, head, batch), query block fastest so that
  // the CTAs running at the same time share a head's K/V through L2.
  __device__ DenseGeo(const DenseParams& prm, int unit) : p(prm) {
    const int qb = unit % p.num_qblocks;
    const int rest = unit / p.num_qblocks;
    q0 = qb * (2 * kBlockM);
    h = rest % p.H;
    b = rest / p.H;
    hk = h / (p.H / p.Hkv);
    int kv = p.Sk;
    if (p.kv_len != nullptr) kv = min(max(p.kv_len[b], 0), p.Sk);
    kv_valid = kv;
  }
  __device__ int num_kv_tiles() const { return (kv_valid + kBlockN - 1) / kBlockN; }
  __device__ bool needs(int, int) const { return true; }
  __device__ bool needs_own(int) const { return true; }
  __device__ int last_tile(int) const { return num_kv_tiles() - 1; }
  __device__ void load_q(const CUtensorMap* tm, int t, uint32_t dst, uint32_t bar,
                         uint64_t pol) const {
#pragma unroll
    for (int c = 0; c < HD / 64; ++c)
      tma_load_4d(dst + c * kHalfBytes, tm, bar, 64 * c, h, q0 + t * kBlockM, b, pol);
  }
  __device__ void load_kv(const CUtensorMap* tm, int j, uint32_t dst, uint32_t bar,
                          uint64_t pol) const {
#pragma unroll
    for (int c = 0; c < HD / 64; ++c)
      tma_load_4d(dst + c * kHalfBytes, tm, bar, 64 * c, hk, j * kBlockN, b, pol);
  }
  __device__ void softmax_setup(int wg, int row) { row_global = q0 + wg * kBlockM + row; }
  // Keys at index >= kv_valid are hidden; every 32-column chunk stays
  // active (the softmax processes all four). cm[c] bit i: column 32c + i.
  __device__ uint32_t chunk_masks(int j, uint32_t (&cm)[4]) const {
    const int rem = kv_valid - j * kBlockN;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int n = rem - c * 32;
      cm[c] = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : (1u << n) - 1u);
    }
    return 0xfu;
  }
  __device__ void apply_masks(const uint32_t (&cm)[4], uint32_t, uint32_t (&sr)[4][32]) const {
    if (cm[3] == 0xffffffffu) return;  // full tile (only the last one can be partial)
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (!((cm[c] >> i) & 1u)) sr[c][i] = 0xff800000u;
  }
  __device__ __nv_bfloat16* row_ptr() const {
    return p.o + b * p.o_sb + static_cast<long long>(row_global) * p.o_ss + h * p.o_sh;
  }
  __device__ void store_row_chunk(int, int, int c, const uint32_t (&pk)[16]) const {
    if (row_global >= p.Sq) return;
    uint4* dst = reinterpret_cast<uint4*>(row_ptr() + c * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
  }
  __device__ void store_zero_row(int, int) const {
    if (row_global >= p.Sq) return;
    uint4* dst = reinterpret_cast<uint4*>(row_ptr());
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
    if (p.lse != nullptr)
      p.lse[(static_cast<long long>(b) * p.H + h) * p.Sq + row_global] = neg_inf();
  }
  __device__ void store_lse(int, int, float lse) const {
    if (p.lse == nullptr || row_global >= p.Sq) return;
    p.lse[(static_cast<long long>(b) * p.H + h) * p.Sq + row_global] = lse;
  }
};

}  // namespace attn
}  // namespace vx

namespace vx {
namespace attn {

// --------------------------------------------------------------------------
// 3-D neighborhood geometry (vidax.models.ltx2_5.diffusion_vae
// .neighborhood_attention_3d, src/vidax/models/ltx2_5/diffusion_vae.py:152-234).
//
// Query (t, h, w) attends the keys in the clamped window
//   [st(t), st(t)+Kt) x [st(h), st(h)+Kh) x [st(w), st(w)+Kw),
//   st(i) = clamp(i - K/2, 0, L - K),  K = min(kernel, L)
// (_window_start, diffusion_vae.py:152-164). Tensors are (B, T, H, W, NH, HD);
// the tensor maps are 5-D {HD, NH, W, H, B*T} (batch and time merged).
//
// A query tile is a box of qt x qh x qw = 128 queries (row order w fastest,
// then h, then t, as TMA writes it); a CTA owns two boxes adjacent along
// `pair_axis`. The CTA visits the key tiles (boxes of KT x KH x KW = 128 keys)
// that tile the union of both boxes' windows; each query tile processes only
// the key tiles that meet its own window union, and masks keys outside each
// query's window. Every window is non-empty, so every valid query sees >= 1
// key.
struct NaParams {
  __nv_bfloat16* o;
  long long o_sb, o_st, o_sh, o_sw, o_shead;  // output strides in elements
  int* status;
  int B, T, H, W, NH, NHkv;
  int kt, kh, kw;          // effective window (kernel clamped to the grid)
  int qbox[3];             // query box (t, h, w), product 128
  int pair_axis;           // 0 = t, 1 = h, 2 = w
  int regions[3];          // CTA regions per axis
  int num_regions;         // regions[0] * regions[1] * regions[2]
  int num_units;           // num_regions * NH * B
  float scale_log2;
  int round_logits;        // round q.k to bf16 before the softmax (vidax's einsum output dtype)
  int o_vec32;             // o and its strides 32-byte aligned: rows stored with 32-byte stores
  // Time slab: q / o hold frames [q_t0, q_t0 + T) and k / v frames
  // [kv_t0, kv_t0 + T_kv) of a T_g-frame grid; windows clamp to the global
  // grid. The unsharded call has T_kv = T_g = T and both offsets 0.
  int T_kv, T_g, q_t0, kv_t0;
};

__device__ __forceinline__ int na_start(int i, int L, int k) {
  return min(max(i - k / 2, 0), L - k);
}

// bits [lo, hi) of an n-bit field (0 <= lo, hi clamped to [0, n])
__device__ __forceinline__ uint32_t bit_range(int lo, int hi, int n) {
  lo = max(lo, 0);
  hi = min(hi, n);
  if (hi <= lo) return 0u;
  const uint32_t upto_hi = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  const uint32_t upto_lo = (1u << lo) - 1u;
  return upto_hi & ~upto_lo;
}

// kHP (head pair): the CTA's two query tiles are one query box of heads h
// and h + 1 instead of two adjacent boxes of one head. Their key unions are
// the same, so every KV step keeps both softmax warpgroups busy (no step
// where only one box needs the key tile), at the price of a K / V tile per
// head in each stage (head_dim 64: 160 KB of shared memory).
template <int KT, int KH, int KW, int HD, bool kHP = false>
struct NaGeo {
  static constexpr int kHeadDim = HD;
  static constexpr bool kPackedSoftmax = true;  // issue-bound (masks): two columns per instruction
  static constexpr int kKVTiles = kHP ? 2 : 1;
  static_assert(KT * KH * KW == 128, "key tile must hold 128 keys");
  static_assert(KW == 8 || KW == 16 || KW == 32, "key tile width 8, 16 or 32");
  using Params = NaParams;
  const NaParams& p;
  int b, head, head_kv;
  int head_kv1;           // kHP: K / V head of query tile 1 (NHkv when that tile is empty)
  bool tile1_valid;       // kHP: head + 1 < NH
  int out_head;           // the softmax thread's query tile's head
  int org[2][3];          // query tile origins
  int lim[3];             // grid extents (T, H, W)
  int u0[3], n_ax[3];     // CTA key union start and tiles per axis
  int wu0[2][3], wu1[2][3];  // per query tile key union [wu0, wu1)
  int n_tiles;
  uint32_t div_w, div_h;  // ceil(2^32 / n_ax[2]), ceil(2^32 / n_ax[1]) (0 for n = 1)
  // softmax row state
  int qc[3];              // query coordinates of this thread's row
  int ws[3];              // window starts
  int own_lo[3], own_hi[3];  // key union of this thread's query tile
  bool row_valid;

  // Work unit u = (region, head, batch), region fastest.
  __device__ NaGeo(const NaParams& prm, int unit) : p(prm) {
    const int rest = unit / p.num_regions;
    if (kHP) {
      const int pairs = (p.NH + 1) / 2;
      head = 2 * (rest % pairs);
      b = rest / pairs;
    } else {
      head = rest % p.NH;
      b = rest / p.NH;
    }
    const int grp = p.NH / p.NHkv;
    head_kv = head / grp;
    tile1_valid = !kHP || head + 1 < p.NH;
    head_kv1 = kHP ? (tile1_valid ? (head + 1) / grp : p.NHkv) : head_kv;
    out_head = head;
    lim[0] = p.T_g;  // window clamping: the global grid
    lim[1] = p.H;
    lim[2] = p.W;
    const int qlim[3] = {p.T, p.H, p.W};  // this call's query frames (local)
    const int qoff[3] = {p.q_t0, 0, 0};   // local -> global query coordinates
    const int ksz[3] = {p.kt, p.kh, p.kw};
    int reg[3];
    int r = unit % p.num_regions;
    reg[2] = r % p.regions[2];
    r /= p.regions[2];
    reg[1] = r % p.regions[1];
    reg[0] = r / p.regions[1];
    const int kvb[3] = {KT, KH, KW};
    int cu0[3] = {0, 0, 0}, cu1[3] = {0, 0, 0};
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int rsz = p.qbox[a] * (a == p.pair_axis ? 2 : 1);
      const int r0 = reg[a] * rsz;
      org[0][a] = r0;
      org[1][a] = r0 + (a == p.pair_axis ? p.qbox[a] : 0);
      bool first = true;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int a0 = org[t][a];
        // kHP: an odd head count leaves the last pair's second tile empty
        const int a1 = (t == 1 && !tile1_valid) ? a0 : min(a0 + p.qbox[a], qlim[a]);
        if (a0 < a1) {
          wu0[t][a] = na_start(a0 + qoff[a], lim[a], ksz[a]);
          wu1[t][a] = na_start(a1 - 1 + qoff[a], lim[a], ksz[a]) + ksz[a];
          if (first) {
            cu0[a] = wu0[t][a];
            cu1[a] = wu1[t][a];
            first = false;
          } else {
            cu0[a] = min(cu0[a], wu0[t][a]);
            cu1[a] = max(cu1[a], wu1[t][a]);
          }
        } else {
          wu0[t][a] = 0;
          wu1[t][a] = 0;  // empty: this query tile lies outside the grid
        }
      }
      u0[a] = cu0[a];
      n_ax[a] = cu1[a] > cu0[a] ? (cu1[a] - cu0[a] + kvb[a] - 1) / kvb[a] : 0;
    }
    n_tiles = n_ax[0] * n_ax[1] * n_ax[2];
    div_w = n_ax[2] > 1 ? 0xffffffffu / static_cast<uint32_t>(n_ax[2]) + 1u : 0u;
    div_h = n_ax[1] > 1 ? 0xffffffffu / static_cast<uint32_t>(n_ax[1]) + 1u : 0u;
  }

  __device__ int num_kv_tiles() const { return n_tiles; }
  // j -> tile origin; quotients by multiply-high with ceil(2^32 / n), exact
  // for j, n < 2^16 (tile counts here are below 2^12).
  __device__ void tile_origin(int j, int (&o)[3]) const {
    const int r = n_ax[2] > 1 ? static_cast<int>(__umulhi(static_cast<uint32_t>(j), div_w)) : j;
    const int jw = j - r * n_ax[2];
    const int jt = n_ax[1] > 1 ? static_cast<int>(__umulhi(static_cast<uint32_t>(r), div_h)) : r;
    const int jh = r - jt * n_ax[1];
    o[0] = u0[0] + jt * KT;
    o[1] = u0[1] + jh * KH;
    o[2] = u0[2] + jw * KW;
  }
  // t may be a run-time value (the softmax warpgroup): selects instead of
  // indexing keep the per-tile arrays in registers.
  __device__ bool needs(int t, int j) const {
    int o[3];
    tile_origin(j, o);
    const int kvb[3] = {KT, KH, KW};
    bool hit = true;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int lo = t ? wu0[1][a] : wu0[0][a];
      const int hi = t ? wu1[1][a] : wu1[0][a];
      hit = hit && (o[a] < hi) && (lo < o[a] + kvb[a]);
    }
    return hit;
  }
  // needs(t, j) for the query tile softmax_setup was given
  __device__ bool needs_own(int j) const {
    int o[3];
    tile_origin(j, o);
    const int kvb[3] = {KT, KH, KW};
    bool hit = true;
#pragma unroll
    for (int a = 0; a < 3; ++a) hit = hit && (o[a] < own_hi[a]) && (own_lo[a] < o[a] + kvb[a]);
    return hit;
  }
  __device__ int last_tile(int t) const {
    for (int j = n_tiles - 1; j >= 0; --j)
      if (needs(t, j)) return j;
    return -1;
  }
  __device__ void load_q(const CUtensorMap* tm, int t, uint32_t dst, uint32_t bar,
                         uint64_t pol) const {
    const int bt = b * p.T + org[t][0];
    const int hq = kHP ? head + t : head;  // an empty tile 1 reads the zero fill past NH
#pragma unroll
    for (int c = 0; c < HD / 64; ++c)
      tma_load_5d(dst + c * kHalfBytes, tm, bar, 64 * c, hq, org[t][2], org[t][1], bt, pol);
  }
  __device__ void load_kv(const CUtensorMap* tm, int j, uint32_t dst, uint32_t bar,
                          uint64_t pol) const {
    int o[3];
    tile_origin(j, o);
    const int bt = b * p.T_kv + (o[0] - p.kv_t0);
#pragma unroll
    for (int c = 0; c < HD / 64; ++c)
      tma_load_5d(dst + c * kHalfBytes, tm, bar, 64 * c, head_kv, o[2], o[1], bt, pol);
    if (kHP) {  // query tile 1's head: the stage's second tile
      constexpr uint32_t kTile = 128u * HD * 2u;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_5d(dst + kTile + c * kHalfBytes, tm, bar, 64 * c, head_kv1, o[2], o[1], bt, pol);
    }
  }
  __device__ void softmax_setup(int t, int row) {
    const int qw = p.qbox[2], qh = p.qbox[1];
    const int iw = row % qw;
    const int ih = (row / qw) % qh;
    const int it = row / (qw * qh);
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      own_lo[a] = t ? wu0[1][a] : wu0[0][a];
      own_hi[a] = t ? wu1[1][a] : wu1[0][a];
    }
    qc[0] = (t ? org[1][0] : org[0][0]) + it;
    qc[1] = (t ? org[1][1] : org[0][1]) + ih;
    qc[2] = (t ? org[1][2] : org[0][2]) + iw;
    row_valid = qc[0] < p.T && qc[1] < p.H && qc[2] < p.W && (t == 0 || tile1_valid);
    out_head = kHP ? head + t : head;
    const int ksz[3] = {p.kt, p.kh, p.kw};
    const int qg[3] = {min(qc[0], p.T - 1) + p.q_t0, qc[1], qc[2]};  // global query coordinates
#pragma unroll
    for (int a = 0; a < 3; ++a) ws[a] = na_start(min(qg[a], lim[a] - 1), lim[a], ksz[a]);
  }
  // Column c of a key tile is key (ct, ch, cw) = (c / (KH*KW), (c / KW) % KH,
  // c % KW) of the tile box; it is visible when each coordinate lies in this
  // row's window. Masks are built per axis as bit fields, then per 32-column
  // chunk (cm[c] bit i: column 32c + i). Returns the chunks (bit c) with a
  // visible column in any row of this warp: the softmax skips the others (no
  // mask, no exponentials; P is zero there).
  //
  // For KW == 16 (the instantiated key tile) every chunk is two (ct, ch) rows
  // of 16 columns that share this row's window columns, so the masks are kept
  // factored: cm[0] = the 16-bit column mask, cm[1] bit r = (ct, ch) row r of
  // the tile (r = ct * KH + ch) is in the window; apply_masks then adds 0 or
  // -inf biases two columns per instruction instead of selecting per column.
  __device__ uint32_t chunk_masks(int j, uint32_t (&cm)[4]) const {
    int o[3];
    tile_origin(j, o);
    const uint32_t tmask = bit_range(ws[0] - o[0], ws[0] + p.kt - o[0], KT);
    const uint32_t hmask = bit_range(ws[1] - o[1], ws[1] + p.kh - o[1], KH);
    const uint32_t wmask = bit_range(ws[2] - o[2], ws[2] + p.kw - o[2], KW);
    constexpr int kRowsPerChunk = 32 / KW;  // (ct, ch) rows of the tile per chunk (>= 1)
    constexpr uint32_t kChunkRows = (1u << kRowsPerChunk) - 1u;
    // factored: cm[0] = the w bits of one tile row, cm[1] bit r = tile row r
    // (r = ct * KH + ch) lies in the window's t and h ranges
    uint32_t rows = 0;
#pragma unroll
    for (int r = 0; r < KT * KH; ++r)
      if (((tmask >> (r / KH)) & 1u) && ((hmask >> (r % KH)) & 1u)) rows |= 1u << r;
    if (!row_valid || wmask == 0u) rows = 0;
    cm[0] = wmask;
    cm[1] = rows;
    cm[2] = cm[3] = 0;
    uint32_t active = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (__any_sync(0xffffffffu, ((rows >> (kRowsPerChunk * c)) & kChunkRows) != 0u))
        active |= 1u << c;
    return active;
  }
  // Hidden columns of the active chunks become -inf (after the optional bf16
  // rounding of q.k); inactive chunks are left as they are.
  // Adds the column bias (0 / -inf by the w bit) and the tile-row bias (0 /
  // -inf by the row bit) to each score, two columns per f32x2 add.
  __device__ void apply_masks(const uint32_t (&cm)[4], uint32_t active,
                              uint32_t (&sr)[4][32]) const {
    constexpr int kRowsPerChunk = 32 / KW;
    const float ninf = neg_inf();
    uint64_t wb[KW / 2];  // column biases of one tile row, two columns per register pair
#pragma unroll
    for (int k = 0; k < KW / 2; ++k)
      wb[k] = f2_pack(((cm[0] >> (2 * k)) & 1u) ? 0.f : ninf,
                      ((cm[0] >> (2 * k + 1)) & 1u) ? 0.f : ninf);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (!((active >> c) & 1u)) continue;
      if (p.round_logits) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          sr[c][i] = __float_as_uint(__bfloat162float(__float2bfloat16_rn(__uint_as_float(sr[c][i]))));
      }
#pragma unroll
      for (int r = 0; r < kRowsPerChunk; ++r) {
        const float rb = ((cm[1] >> (kRowsPerChunk * c + r)) & 1u) ? 0.f : ninf;
        const uint64_t rb2 = f2_pack(rb, rb);
#pragma unroll
        for (int k = 0; k < KW / 2; ++k) {
          const int i = KW * r + 2 * k;
          float a, bq;
          f2_unpack(f2_add(f2_add(f2_pack(__uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1])),
                                  wb[k]), rb2), a, bq);
          sr[c][i] = __float_as_uint(a);
          sr[c][i + 1] = __float_as_uint(bq);
        }
      }
    }
  }
  __device__ __nv_bfloat16* row_ptr() const {
    return p.o + b * p.o_sb + qc[0] * p.o_st + qc[1] * p.o_sh + qc[2] * p.o_sw +
           out_head * p.o_shead;
  }
  // A warp's 32 rows are 32 different output rows (neighbouring w are a whole
  // token apart), so each store touches 32 lines: 32-byte stores write whole
  // sectors (half as many L2 writes as 16-byte stores; 3 % faster on cfg4
  // than 16-byte stores, and faster than staging the rows through shared
  // memory for 128-byte coalesced stores, which lengthened the epilogue).
  __device__ void store_row_chunk(int, int, int c, const uint32_t (&pk)[16]) const {
    if (!row_valid) return;
    __nv_bfloat16* dst = row_ptr() + c * 32;
    if (p.o_vec32) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        st_global_v8(dst + 16 * i, pk[8 * i], pk[8 * i + 1], pk[8 * i + 2], pk[8 * i + 3],
                     pk[8 * i + 4], pk[8 * i + 5], pk[8 * i + 6], pk[8 * i + 7]);
    } else {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
    }
  }
  __device__ void store_zero_row(int, int) const {
    if (!row_valid) return;
    uint4* dst = reinterpret_cast<uint4*>(row_ptr());
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
  }
  __device__ void store_lse(int, int, float) const {}
};

}  // namespace attn
}  // namespace vx
