// gemm_tn_sm100.cu -- the sibling GEMM families the reference drives through
// the same client (client/aiter/hsa/gfx942/gemm_driver.py), on B200 (sm_100a):
//
//   BF16 TN          Y[m,n] = bf16( sum_k A[m,k] * B[n,k]  (+ bias[n]) )
//                    (gemm_driver.py:50: (a.float() @ b.float().T).bfloat16())
//   INT8 per token   Y[m,n] = bf16( float(sum_k A[m,k] * B[n,k]) * sa[m] * sb[n] + bias[n] )
//                    (gemm_driver.py:73: ((a.float() @ b.float().T) * sa * sb.T + bias))
//
// Unlike the block-scaled FP8 path, nothing rescales between K blocks, so the
// whole K range of a tile accumulates inside TMEM and the epilogue runs once:
//  * a CTA owns a 128-row x BN-column tile (BN = 64, 128, 256): rows are the
//    UMMA M side (TMEM lanes), columns the N side (TMEM columns, BN of them);
//    or (PAIR) two CTAs of a cluster share a 256-row x BN tile through
//    tcgen05 cta_group::2: each loads its own 128 rows of A and half of the BN
//    rows of B, the even CTA issues the M = 256 MMA and each receives its 128
//    accumulator rows in its own TMEM -- B bytes per CTA halve, and since the
//    accumulator stays in TMEM for the whole K range the only per-chunk
//    handshake is the commit that frees both CTAs' stages;
//  * warp 0 (one thread) streams 128-byte K chunks of both operands (64 bf16
//    or 128 int8 elements) into a 4-8 stage mbarrier ring with TMA (128-byte
//    swizzle; the pre-packed weight layout of the FP8 path applies unchanged to
//    these bytes); warp 1 (one thread) issues 4 tcgen05.mma per chunk --
//    kind::f16 (K = 16) or kind::i8 (K = 32, exact s32 accumulation) -- and one
//    commit per chunk to free its stage, then one commit for the finished
//    accumulator;
//  * warps 2-5 read the accumulator with tcgen05.ld (one row per thread),
//    apply the scales and bias in the reference's operation order
//    ((acc * sa) * sb + bias, each rounded in fp32, no fused multiply-add) and
//    store bf16 rows;
//  * split-K (small M): the K slices of a tile form a thread-block cluster
//    along z; each CTA stages its raw accumulator (fp32 or s32) in its idle
//    stage ring and sums a disjoint block of rows over all slices through
//    distributed shared memory in slice order 0..S-1 (int32 sums for INT8:
//    exact; fp32 sums for BF16: bitwise reproducible);
//  * every mbarrier wait is bounded (the library's status word records an
//    expiry); no TMA multicast.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/fack_gemm.h"
#include "fack_internal.h"
#include "sm100_ptx.cuh"
#include "tuned_table.h"

namespace fack_tn {

using namespace fack;

constexpr int kTileM = 128;
constexpr int kChunk = 128;          // bytes of K per stage: one 128-byte swizzle row
constexpr int kThreads = 192;        // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kMaxSplit = 8;         // portable cluster size
constexpr int kGroupM = 16;          // row-tile band of the grouped launch order
constexpr int kSmemBudget = 196608;
constexpr unsigned kStTn = 128u;     // status flag: a wait in the sibling GEMM gave up

template <int BN, bool PAIR>
struct TnCfg {
  static_assert(BN == 64 || BN == 128 || BN == 256, "column tile must be 64, 128 or 256");
  static constexpr int kBRows = PAIR ? BN / 2 : BN;  // B rows this CTA loads per chunk
  static constexpr int kABytes = kTileM * kChunk;    // 16 KB
  static constexpr int kBBytes = kBRows * kChunk;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr int kPitch = BN + 4;             // 32-bit words per staged row (split-K)
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kStages * kABytes;
  static constexpr int kOffBar = kOffB + kStages * kBBytes;
  static constexpr int kNumBars = 2 * kStages + 2;  // full, empty, accumulator, drain
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;
  static_assert(kStages >= 2, "pipeline needs two stages");
  static_assert(kTileM * kPitch * 4 <= kOffBar, "split-K staging must fit in the stage ring");
};

struct TnParams {
  const float* a_scale;   // [M], INT8 only
  const float* b_scale;   // [N], INT8 only
  const float* bias;      // [N] or NULL
  __nv_bfloat16* out;
  int64_t ldo;
  int M, N, KC;           // KC = K bytes / 128
  int split;
  int b_packed;
  unsigned int* status;
  uint64_t timeout_ns;
};

// One output element from the raw accumulator bits.
template <int KIND>
__device__ __forceinline__ float finish(uint32_t bits, float sa, float sb, const float* bias, int n) {
  float v;
  if constexpr (KIND == FACK_GEMM_I8)
    v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(bits)), sa), sb);
  else
    v = __uint_as_float(bits);
  return bias ? __fadd_rn(v, __ldg(bias + n)) : v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

template <int KIND, int BN, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_a,
               const __grid_constant__ TnParams p) {
  using C = TnCfg<BN, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // grid: single CTAs (x = column tile, y = 128-row tile); pairs (x = 128-row
  // tile, an even count so a pair lies along the cluster's x, y = column
  // tile); z = K slice.  Grouped launch order: consecutive CTAs walk a band of
  // kGroupM row-tile slots before the next column tile, so co-resident CTAs
  // share operands in L2.
  int mt, nt;
  {
    const int unit = PAIR ? 2 : 1;
    const int m_slots = PAIR ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.y);
    const int n_tiles = PAIR ? static_cast<int>(gridDim.y) : static_cast<int>(gridDim.x);
    const int lin = PAIR ? static_cast<int>(blockIdx.x) / 2 + static_cast<int>(blockIdx.y) * m_slots
                         : static_cast<int>(blockIdx.x) + static_cast<int>(blockIdx.y) * n_tiles;
    const int per_group = kGroupM * n_tiles;
    const int g = lin / per_group;
    const int first = g * kGroupM;
    const int gm = min(kGroupM, m_slots - first);
    const int r = lin - g * per_group;
    nt = r / gm;
    mt = (first + r % gm) * unit + (PAIR ? static_cast<int>(blockIdx.x & 1) : 0);
  }
  const int s = blockIdx.z;
  const int S = p.split;
  const int m0 = mt * kTileM;
  const int n0 = nt * BN;
  const int kc0 = (s * p.KC) / S;
  const int nk = ((s + 1) * p.KC) / S - kc0;
  const int rows = min(kTileM, p.M - m0);   // may be <= 0 for a pair's second CTA
  // pair bookkeeping: cluster dims (2, 1, S), rank = (mt & 1) + 2 * s
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = !PAIR || (mt & 1) == 0;
  const uint32_t leader_rank = crank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader_rank);

  const uint32_t bar0 = base + C::kOffBar;
  auto bar_full = [&](int i) { return bar0 + 8u * i; };
  auto bar_empty = [&](int i) { return bar0 + 8u * (C::kStages + i); };
  const uint32_t bar_acc = bar0 + 8u * (2 * C::kStages);
  const uint32_t bar_drain = bar_acc + 8u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(bar_full(i), 1);
      mbar_init(bar_empty(i), 1);
    }
    mbar_init(bar_acc, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_addr(tmem_slot), BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_addr(tmem_slot), BN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();  // both CTAs' barriers are initialised before either signals the other's
  } else {
    __syncthreads();
  }
  tc_fence_after();
  grid_dependency_wait();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t tmo = p.timeout_ns;
  unsigned int* status = p.status;
  int produced = 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const uint64_t pol_b = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        if (!wait_bounded(bar_empty(st), ph ^ 1u, abort_flag, status, kStTn, tmo)) break;
        const int kc = kc0 + i;
        const uint32_t sa = base + C::kOffA + st * C::kABytes;
        const uint32_t sb = base + C::kOffB + st * C::kBBytes;
        const int br0 = n0 + (PAIR ? static_cast<int>(mt & 1) * C::kBRows : 0);  // first B row loaded here
        if constexpr (PAIR) {
          // both CTAs' bytes complete on the leader's full barrier
          const uint32_t fb = dsmem_map(bar_full(st), leader_rank);
          if (leader) mbar_arrive_expect_tx(bar_full(st), 2 * C::kStageBytes);
          tma_load_2d_pair(sa, &tmap_a, fb, kc * kChunk, m0, pol_a);
          if (p.b_packed) {
#pragma unroll
            for (int t = 0; t < (C::kBRows + 127) / 128; ++t)
              tma_load_2d_pair(sb + t * 16384, &tmap_b, fb, 0, (((br0 >> 7) + t) * p.KC + kc) * 128 + (br0 & 127),
                               pol_b);
          } else {
            tma_load_2d_pair(sb, &tmap_b, fb, kc * kChunk, br0, pol_b);
          }
        } else {
          mbar_arrive_expect_tx(bar_full(st), C::kStageBytes);
          tma_load_2d(sa, &tmap_a, bar_full(st), kc * kChunk, m0, pol_a);
          if (p.b_packed) {
#pragma unroll
            for (int t = 0; t < (C::kBRows + 127) / 128; ++t)
              tma_load_2d(sb + t * 16384, &tmap_b, bar_full(st), 0, (((br0 >> 7) + t) * p.KC + kc) * 128 + (br0 & 127),
                          pol_b);
          } else {
            tma_load_2d(sb, &tmap_b, bar_full(st), kc * kChunk, br0, pol_b);
          }
        }
        produced = i + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0 && leader) {
      constexpr int kMmaM = PAIR ? 2 * kTileM : kTileM;
      constexpr uint32_t idesc = KIND == FACK_GEMM_I8 ? idesc_s8_s32(kMmaM, BN) : idesc_bf16_f32(kMmaM, BN);
      int i = 0;
      for (; i < nk; ++i) {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        if (!wait_bounded(bar_full(st), ph, abort_flag, status, kStTn, tmo)) break;
        tc_fence_after();
        const uint64_t da = sw128_kmajor_desc(base + C::kOffA + st * C::kABytes);
        const uint64_t db = sw128_kmajor_desc(base + C::kOffB + st * C::kBBytes);
#pragma unroll
        for (int k = 0; k < kChunk / 32; ++k) {  // 32 bytes of K per MMA = 2 descriptor units
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          if constexpr (PAIR && KIND == FACK_GEMM_I8)
            umma_s8_pair(tmem_base, da + 2 * k, db + 2 * k, idesc, acc);
          else if constexpr (PAIR)
            umma_bf16_pair(tmem_base, da + 2 * k, db + 2 * k, idesc, acc);
          else if constexpr (KIND == FACK_GEMM_I8)
            umma_s8(tmem_base, da + 2 * k, db + 2 * k, idesc, acc);
          else
            umma_bf16(tmem_base, da + 2 * k, db + 2 * k, idesc, acc);
        }
        if constexpr (PAIR)
          umma_commit_pair_mc(bar_empty(st), pair_mask);  // frees the stage in both CTAs
        else
          umma_commit(bar_empty(st));
      }
      if (i == nk) {  // the whole K range of this slice is in TMEM
        if constexpr (PAIR)
          umma_commit_pair_mc(bar_acc, pair_mask);
        else
          umma_commit(bar_acc);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;     // tile row of this thread
    const bool got = wait_bounded(bar_acc, 0, abort_flag, status, kStTn, tmo);
    if (__all_sync(0xffffffffu, got)) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      const bool valid = row < rows;
      float sa = 1.0f;
      if constexpr (KIND == FACK_GEMM_I8) sa = valid ? __ldg(p.a_scale + m0 + row) : 0.0f;
      __nv_bfloat16* orow = p.out + static_cast<int64_t>(m0 + (valid ? row : 0)) * p.ldo + n0;
      uint32_t* srow = reinterpret_cast<uint32_t*>(smem + C::kOffA) + row * C::kPitch;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(taddr + c * 32, v);
        if (S > 1) {
          // raw accumulator bits into the idle stage ring (every stage was
          // consumed by an MMA that completed before bar_acc fired)
#pragma unroll
          for (int t = 0; t < 32; t += 4)
            *reinterpret_cast<uint4*>(srow + c * 32 + t) = make_uint4(v[t], v[t + 1], v[t + 2], v[t + 3]);
        } else if (valid) {
          uint32_t pk[16];
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            const int n = n0 + c * 32 + t;
            float sb0 = 1.0f, sb1 = 1.0f;
            if constexpr (KIND == FACK_GEMM_I8) {
              sb0 = __ldg(p.b_scale + n);
              sb1 = __ldg(p.b_scale + n + 1);
            }
            pk[t / 2] = pack_bf16x2(finish<KIND>(v[t], sa, sb0, p.bias, n), finish<KIND>(v[t + 1], sa, sb1, p.bias, n + 1));
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int t = 0; t < 4; ++t) dst[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown --
  grid_launch_dependents();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    if (*abort_flag && lane == 0) {
      // wait (bounded, fresh deadline) for the copies issued, so none lands after exit
      const int first = produced > C::kStages ? produced - C::kStages : 0;
      volatile int no_abort = 0;
      if (leader) {
        for (int i = first; i < produced; ++i)
          wait_bounded(bar_full(i % C::kStages), (i / C::kStages) & 1, &no_abort, status, kStTn, tmo);
      } else {
        // a pair's second CTA signals its loads on the leader's barrier and
        // cannot observe them: give them a bounded 50 us to land
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 50000u) __nanosleep(1000);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // arrives once every MMA of this thread has completed
      if constexpr (PAIR)
        umma_commit_pair(bar_drain);
      else
        umma_commit(bar_drain);
      volatile int no_abort = 0;
      wait_bounded(bar_drain, 0, &no_abort, status, kStTn, tmo);
    }
    __syncwarp();
  }
  if constexpr (PAIR) {
    // the leader's MMAs have drained and the peer's loads were consumed (or
    // drained): only now may either CTA free its TMEM
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, BN);
    else
      tmem_dealloc(tmem_base, BN);
  }
  if (S == 1) return;

  // Split-K over distributed shared memory.  Every CTA of the cluster reaches
  // both barriers, also after an abort; the second keeps each CTA's staging
  // alive until every peer has read it.
  const bool ok = *abort_flag == 0;
  const int rows_v = rows > 0 ? rows : 0;
  const int per = (rows_v + S - 1) / S;
  const int r0 = s * per;
  const int r1 = min(rows_v, r0 + per);
  const int rank_step = PAIR ? 2 : 1;            // cluster rank of slice t: rank0 + rank_step * t
  const int rank0 = PAIR ? static_cast<int>(mt & 1) : 0;
  cluster_sync_all();
  if (ok) {
    constexpr int kRowQ = BN / 4;
    const uint32_t stg = base + C::kOffA;
    const int items = (r1 > r0 ? r1 - r0 : 0) * kRowQ;
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int r = r0 + it / kRowQ;
      const int c = (it % kRowQ) * 4;
      const uint32_t addr = stg + static_cast<uint32_t>((r * C::kPitch + c) * 4);
      float out4[4];
      if constexpr (KIND == FACK_GEMM_I8) {
        int acc[4] = {0, 0, 0, 0};
        for (int t = 0; t < S; ++t) {
          const float4 f = dsmem_ld4(dsmem_map(addr, rank0 + rank_step * t));
          acc[0] += __float_as_int(f.x);
          acc[1] += __float_as_int(f.y);
          acc[2] += __float_as_int(f.z);
          acc[3] += __float_as_int(f.w);
        }
        const float sa = __ldg(p.a_scale + m0 + r);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          out4[j] = finish<KIND>(static_cast<uint32_t>(acc[j]), sa, __ldg(p.b_scale + n0 + c + j), p.bias, n0 + c + j);
      } else {
        float4 sum = dsmem_ld4(dsmem_map(addr, rank0));
        for (int t = 1; t < S; ++t) {
          const float4 f = dsmem_ld4(dsmem_map(addr, rank0 + rank_step * t));
          sum.x += f.x;
          sum.y += f.y;
          sum.z += f.z;
          sum.w += f.w;
        }
        const float raw[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) out4[j] = finish<KIND>(__float_as_uint(raw[j]), 1.0f, 1.0f, p.bias, n0 + c + j);
      }
      *reinterpret_cast<uint2*>(p.out + static_cast<int64_t>(m0 + r) * p.ldo + n0 + c) =
          make_uint2(pack_bf16x2(out4[0], out4[1]), pack_bf16x2(out4[2], out4[3]));
    }
  }
  cluster_sync_all();
}

// ===================================================================== host ==

constexpr int kVariants = 12;  // (bf16, i8) x (64, 128, 256) x (single CTA, CTA pair)
constexpr int kMaxDevices = 64;

static int variant(int kind, int tm, int bn) {
  return kind * 6 + (tm == 256 ? 3 : 0) + (bn == 64 ? 0 : bn == 128 ? 1 : 2);
}

struct Entry {
  const void* fn;
  int smem;
};

template <int KIND, int BN, bool PAIR>
static Entry entry() {
  return {reinterpret_cast<const void*>(gemm_tn_kernel<KIND, BN, PAIR>), TnCfg<BN, PAIR>::kSmemBytes};
}

static const Entry& kernel_for(int kind, int tm, int bn) {
  static const Entry table[kVariants] = {
      entry<FACK_GEMM_BF16, 64, false>(), entry<FACK_GEMM_BF16, 128, false>(), entry<FACK_GEMM_BF16, 256, false>(),
      entry<FACK_GEMM_BF16, 64, true>(),  entry<FACK_GEMM_BF16, 128, true>(),  entry<FACK_GEMM_BF16, 256, true>(),
      entry<FACK_GEMM_I8, 64, false>(),   entry<FACK_GEMM_I8, 128, false>(),   entry<FACK_GEMM_I8, 256, false>(),
      entry<FACK_GEMM_I8, 64, true>(),    entry<FACK_GEMM_I8, 128, true>(),    entry<FACK_GEMM_I8, 256, true>()};
  return table[variant(kind, tm, bn)];
}

struct DevState {
  unsigned configured = 0;
  int clusters[kVariants][kMaxSplit + 1] = {};
};

static std::mutex g_mu;
static DevState g_dev[kMaxDevices];

static int dev_state(DevState** out, int* sms) {
  const int st = sm100_device(sms);
  if (st != FACK_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FACK_ERR_CUDA;
  *out = &g_dev[dev];
  return FACK_OK;
}

static int configure(DevState* d, int kind, int tm, int bn) {
  const int v = variant(kind, tm, bn);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!(d->configured & (1u << v))) {
    const Entry& k = kernel_for(kind, tm, bn);
    const cudaError_t e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
    if (e != cudaSuccess) return record_error(FACK_ERR_LAUNCH, "cudaFuncSetAttribute(sibling GEMM shared memory)");
    d->configured |= 1u << v;
  }
  return FACK_OK;
}

// Clusters of (tm/128, 1, split) CTAs of a variant the device holds at once
// (a cluster must fit inside one GPC).
static int co_resident(DevState* d, int sms, int kind, int tm, int bn, int split) {
  const int v = variant(kind, tm, bn);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (d->clusters[v][split]) return d->clusters[v][split];
  }
  if (configure(d, kind, tm, bn) != FACK_OK) return 0;
  const Entry& k = kernel_for(kind, tm, bn);
  const int cx = tm / kTileM;
  int n = 0;
  if (split == 1 && cx == 1) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k.fn, kThreads, k.smem) != cudaSuccess) return 0;
    n = per_sm * sms;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cx, 1, split);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = k.smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cx;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = split;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, k.fn, &cfg) != cudaSuccess) return 0;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  d->clusters[v][split] = n;
  return n;
}

static int elem_bytes(int kind) { return kind == FACK_GEMM_BF16 ? 2 : 1; }

static int check_shape(int kind, int M, int N, int K) {
  if (kind != FACK_GEMM_BF16 && kind != FACK_GEMM_I8) return FACK_ERR_BAD_ARG;
  const int64_t kbytes = static_cast<int64_t>(K) * elem_bytes(kind);
  if (M < 1 || M > 65535 * kTileM || N < 64 || N % 64 || K < 1 || kbytes % kChunk || kbytes > (1ll << 30))
    return FACK_ERR_BAD_SHAPE;
  return FACK_OK;
}

// Grid of a plan.  Single CTAs: x = column tiles, y = 128-row tiles.  Pairs:
// x = 128-row tiles (an even count; a pair's second CTA may hold no valid
// row), y = column tiles.  z = K slices.
static dim3 plan_grid(int M, int N, int tm, int bn, int sp) {
  if (tm == 256) return dim3(2 * ((M + 255) / 256), N / bn, sp);
  return dim3(N / bn, (M + kTileM - 1) / kTileM, sp);
}

// Estimated cycles of a plan (the same per-SM rates as the block-scaled
// planner, without its per-K-block rescale): per 128-byte K chunk the slower
// of the TMA fill (~44 B/clk of A rows plus this CTA's B rows) and the MMA
// (2*bn cycles for 128 rows), plus ~3000 cycles per CTA (a pair: ~1000 more
// for its cluster handshakes) and the output (bf16 stores ~24 B/clk, or the
// split-K exchange ~18 B/clk and two cluster barriers), times the waves of
// co-resident clusters; floored by the HBM time of the operands.
static double plan_cost(DevState* d, int sms, int kind, int M, int N, int K, int tm, int bn, int sp) {
  const int KC = static_cast<int>(static_cast<int64_t>(K) * elem_bytes(kind) / kChunk);
  const dim3 g = plan_grid(M, N, tm, bn, sp);
  const int ctas = static_cast<int>(g.x * g.y);                   // CTAs per K slice
  const int slots = co_resident(d, sms, kind, tm, bn, sp) * (tm / kTileM);
  if (slots <= 0) return 1e30;
  const int waves = (ctas + slots - 1) / slots;
  const int steps = (KC + sp - 1) / sp;
  const int rows = M < kTileM ? M : kTileM;
  const double brows = tm == 256 ? bn / 2.0 : bn;
  const double t_chunk = fmax((kTileM * 128.0 + brows * 128.0) / 44.0, 2.0 * bn);
  const double out = sp > 1 ? rows * bn * 4.0 * (sp - 1) / sp / 18.0 + 2500.0 : rows * bn * 2.0 / 24.0;
  const double fixed = tm == 256 ? 4000.0 : 3000.0;
  const double cyc = static_cast<double>(waves) * (steps * t_chunk + fixed + out);
  const double bytes = (static_cast<double>(N) + M) * K * elem_bytes(kind);
  return fmax(cyc, bytes / 6.5e12 * 1.9e9);
}

}  // namespace fack_tn

using namespace fack_tn;

extern "C" {

int fack_gemm_tn_plan(int kind, int M, int N, int K, int tile_m_request, int tile_n_request, int split_k_request,
                      int* tile_m, int* tile_n, int* split_k) {
  int st = check_shape(kind, M, N, K);
  if (st != FACK_OK) return st;
  if (!tile_m || !tile_n || !split_k) return FACK_ERR_BAD_ARG;
  const int KC = static_cast<int>(static_cast<int64_t>(K) * elem_bytes(kind) / kChunk);
  if (tile_m_request != 0 && tile_m_request != 128 && tile_m_request != 256) return FACK_ERR_BAD_ARG;
  if (tile_n_request != 0 && tile_n_request != 64 && tile_n_request != 128 && tile_n_request != 256)
    return FACK_ERR_BAD_ARG;
  if (tile_n_request && N % tile_n_request) return FACK_ERR_BAD_ARG;
  if (split_k_request < 0 || split_k_request > kMaxSplit || split_k_request > KC) return FACK_ERR_BAD_ARG;
  if (tile_m_request == 256 && 2 * split_k_request > kMaxSplit) return FACK_ERR_BAD_ARG;  // cluster of 2 x split
  if (tile_m_request && tile_n_request && split_k_request) {
    *tile_m = tile_m_request;
    *tile_n = tile_n_request;
    *split_k = split_k_request;
    return FACK_OK;
  }
  DevState* d = nullptr;
  int sms = 0;
  st = dev_state(&d, &sms);
  if (st != FACK_OK) return st;
  // an exact-shape row of the sibling table fixes a fully automatic plan
  if (!tile_m_request && !tile_n_request && !split_k_request &&
      fack::tn_tuned_lookup(kind, sms, M, N, K, tile_m, tile_n, split_k))
    return FACK_OK;
  double best = 1e30;
  int bt = 0, bb = 0, bs = 0;
  for (int tm : {128, 256}) {
    if (tile_m_request && tm != tile_m_request) continue;
    for (int bn : {256, 128, 64}) {
      if (N % bn || (tile_n_request && bn != tile_n_request)) continue;
      for (int sp = 1; sp <= KC && sp * (tm / kTileM) <= kMaxSplit; ++sp) {
        if (split_k_request && sp != split_k_request) continue;
        if (!split_k_request && sp > 1 && KC / sp < 2) break;
        const double c = plan_cost(d, sms, kind, M, N, K, tm, bn, sp);
        if (c < best * 0.97) {  // prefer the earlier candidate unless clearly faster
          best = c;
          bt = tm;
          bb = bn;
          bs = sp;
        }
      }
    }
  }
  if (!bb) return FACK_ERR_LAUNCH;
  *tile_m = bt;
  *tile_n = bb;
  *split_k = bs;
  return FACK_OK;
}

int fack_gemm_tn(int kind, const void* a, int64_t lda, const void* b, int b_packed, int64_t ldb,
                 const float* a_scale, const float* b_scale, const float* bias, void* out, int64_t ldo, int M,
                 int N, int K, int tile_m, int tile_n, int split_k, void* stream) {
  int st = check_shape(kind, M, N, K);
  if (st != FACK_OK) return st;
  if (b_packed != 0 && b_packed != 1) return FACK_ERR_BAD_ARG;
  const int es = elem_bytes(kind);
  auto al = [](const void* ptr, uintptr_t n) { return ptr && reinterpret_cast<uintptr_t>(ptr) % n == 0; };
  if (!al(a, 16) || !al(b, 16) || !al(out, 16)) return FACK_ERR_BAD_ALIGN;
  if (kind == FACK_GEMM_I8) {
    if (!al(a_scale, 4) || !al(b_scale, 4)) return FACK_ERR_BAD_ALIGN;
  } else if (a_scale || b_scale) {
    return FACK_ERR_BAD_ARG;  // the BF16 family has no scales
  }
  if (bias && !al(bias, 4)) return FACK_ERR_BAD_ALIGN;
  if (lda < K || (lda * es) % 16 || ldo < N || ldo % 8) return FACK_ERR_BAD_STRIDE;
  if (!b_packed && (ldb < K || (ldb * es) % 16)) return FACK_ERR_BAD_STRIDE;
  int tm = 0, bn = 0, sp = 0;
  st = fack_gemm_tn_plan(kind, M, N, K, tile_m, tile_n, split_k, &tm, &bn, &sp);
  if (st != FACK_OK) return st;

  DevState* d = nullptr;
  int sms = 0;
  st = dev_state(&d, &sms);
  if (st != FACK_OK) return st;
  st = configure(d, kind, tm, bn);
  if (st != FACK_OK) return st;

  const uint64_t kbytes = static_cast<uint64_t>(K) * es;
  const int KC = static_cast<int>(kbytes / kChunk);
  const uint32_t brows = tm == 256 ? bn / 2 : bn;  // B rows one CTA loads
  CUtensorMap ta, tb;
  st = encode_bytes_2d(&ta, a, kbytes, static_cast<uint64_t>(M), static_cast<uint64_t>(lda) * es, kChunk, kTileM, true);
  if (st != FACK_OK) return st;
  if (b_packed)
    st = encode_bytes_2d(&tb, b, kChunk, static_cast<uint64_t>(N) * KC, kChunk, kChunk, brows < 128 ? brows : 128, false);
  else
    st = encode_bytes_2d(&tb, b, kbytes, static_cast<uint64_t>(N), static_cast<uint64_t>(ldb) * es, kChunk, brows, true);
  if (st != FACK_OK) return st;
  unsigned int* status = device_status_word();
  if (!status) return record_error(FACK_ERR_CUDA, "status word address");

  TnParams p;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.bias = bias;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.M = M;
  p.N = N;
  p.KC = KC;
  p.split = sp;
  p.b_packed = b_packed;
  p.status = status;
  p.timeout_ns = 2000000000ull;

  const Entry& k = kernel_for(kind, tm, bn);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = plan_grid(M, N, tm, bn, sp);
  if (cfg.gridDim.y > 65535 || cfg.gridDim.z > 65535) return FACK_ERR_BAD_SHAPE;  // beyond one launch's grid
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = k.smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
  ++cfg.numAttrs;
  if (sp > 1 || tm == 256) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = tm / kTileM;  // pairs lie along cluster x
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = sp;
    ++cfg.numAttrs;
  }
  void* args[] = {&tb, &ta, &p};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, k.fn, args);
  if (e != cudaSuccess) return record_error(FACK_ERR_LAUNCH, cudaGetErrorName(e));
  return FACK_OK;
}

}  // extern "C"
