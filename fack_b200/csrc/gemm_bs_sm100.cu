// gemm_bs_sm100.cu -- FP8 (e4m3) block-scaled GEMM for B200 (sm_100a).
//
//   Y[m,n] (bf16) = sum_kb (XQ[m,kb-block] . WQ[n,kb-block]) * x_scale[m,kb] * w_scale[n/128,kb]
//
// The arithmetic restated from client/aiter/hsa/gfx942/driver.py:18-20 (the
// reference's fp32 oracle for aiter's gemm_a8w8_blockscale_bpreshuffle_asm).
//
// Design (B200-first, not a translation of the gfx942 kernels):
//  * a CTA owns a 128-token x BN-weight-row output tile (BN = 64/128/256):
//    the tokens are the UMMA M side (TMEM lanes), the weight rows the UMMA N
//    side (TMEM columns).  Each thread of the rescale warps owns one token,
//    so the per-K-block scale it needs is one scalar,
//    x_scale[m,kb] * w_scale[n/128,kb] (two for a 256-row tile, one per half).
//  * per 128-wide K block (kb): TMA brings the 128x128 B token tile and the
//    BNx128 B weight tile into a multi-stage mbarrier ring (128-byte
//    swizzle); one thread issues 4 tcgen05.mma (K=32 each) into one of 2-4
//    TMEM buffers; 8 rescale warps (two per TMEM lane quarter) read the
//    finished buffer with tcgen05.ld and fold it into fp32 register
//    accumulators, acc += partial * scale -- the per-block rescale cannot go
//    into the MMA because the scales are arbitrary fp32 values, not UE8M0
//    powers of two.  Several TMEM buffers let the MMA run ahead of the
//    rescale.  Warpgroup 0 (TMA, MMA) gives registers to the two rescale
//    warpgroups with setmaxnreg.  Scales are prefetched a few K blocks ahead
//    with cp.async into per-thread shared slots.
//  * split-K for small M: the K slices of one output tile form a thread-block
//    cluster along grid z.  Each CTA writes its fp32 partial tile to the
//    workspace, the cluster barrier publishes them, and each CTA then sums a
//    disjoint set of rows over all slices in slice order 0..S-1, so results
//    are bitwise reproducible and no CTA ever spins on another.
//  * outputs (bf16 tile or fp32 partial) are staged in shared memory with a
//    padded pitch and written with coalesced 16-byte stores.
//  * every mbarrier wait is bounded by a %globaltimer deadline; on expiry the
//    CTA raises an abort flag, records a code in the device status word,
//    drains its in-flight TMA copies and MMAs, frees TMEM and exits.
//  * no TMA multicast anywhere: the same kernel serves the N-sharded
//    multi-GPU path.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <type_traits>

#include "../../include/fack_gemm.h"
#include "sm100_ptx.cuh"
#include "tuned_table.h"

namespace fack {

constexpr int kBlk = 128;          // quantisation block along K and N
constexpr int kTileM = 128;        // tokens per CTA (UMMA M, TMEM lanes)
constexpr int kMaxM = 65535 * 128; // token tiles ride on gridDim.y (at most 65535)
constexpr int kThreads = 384;      // 12 warps = 3 warpgroups
constexpr int kEpiWarp0 = 4;       // warpgroup 0: TMA, MMA, 2 spare; warps 4..11 rescale and store
constexpr int kPrefetch = 4;       // K blocks of scales prefetched ahead by cp.async
constexpr int kMaxSplit = 8;       // portable cluster size
constexpr int kSwapMaxKb = 128;    // swapped small-M tiles: K blocks per CTA whose scales fit in shared memory
constexpr int kSmallRows = 16;     // weight rows per CTA of the warp-MMA small-M kernel (its plans' tile_n)
constexpr int kSmallMaxKb = 256;   // warp-MMA small-M kernel: K blocks whose scale table fits in shared memory
constexpr int kGroupM = 16;        // token-tile band of the grouped launch order
constexpr int kSmemBudget = 196608;
// Register split (setmaxnreg).  The kernel is launched with kLaunchRegs per
// thread (ptxas' cap for 384 threads, 3 warps per scheduler); warpgroup 0
// gives registers back and warpgroups 1-2 take them.  Per scheduler: one
// control warp + two rescale warps = kCtrlRegs + 2 * kEpiRegs <= 3 * kLaunchRegs.
constexpr int kLaunchRegs = 168;
constexpr int kCtrlRegs = 72;
constexpr int kEpiRegs = 216;
static_assert(kCtrlRegs + 2 * kEpiRegs <= 3 * kLaunchRegs, "register split exceeds the launch allocation");
static_assert(kCtrlRegs % 8 == 0 && kEpiRegs % 8 == 0, "setmaxnreg counts are multiples of 8");

// Device status word: set by kernels whose bounded waits expired.
__device__ unsigned int g_status;

enum : unsigned int {
  kStProducer = 1u,
  kStMma = 2u,
  kStEpilogue = 8u,
  kStDrain = 16u
};

template <int BN, bool PAIR>
struct Cfg {
  static_assert(BN == 64 || BN == 128 || BN == 256, "weight tile must be 64, 128 or 256 rows");
  static constexpr int kWRows = PAIR ? BN / 2 : BN;         // weight rows this CTA loads per K block
  static constexpr int kABytes = kTileM * kBlk;             // 16 KB token tile
  static constexpr int kBBytes = kWRows * kBlk;             // weight tile (this CTA's part)
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr int kTmemBufs = (512 / BN) > 4 ? 4 : (512 / BN);
  static constexpr int kTmemCols = kTmemBufs * BN;          // 512, 512, 256: powers of two
  static constexpr int kCpw = BN / 2;                       // columns per rescale warp
  static constexpr int kPitch32 = BN + 4;                   // fp32 staging pitch (floats)
  static constexpr int kPitch16 = BN + 8;                   // bf16 staging pitch (elements)
  // paired fp32 FMA (fma.rn.f32x2) in the rescale: half the instructions; the
  // 128-wide tiles keep scalar FMAs, with which their registers fit unspilled
  // (with paired FMAs they spill, whether TMEM is read 16 or 32 columns at a time)
  static constexpr bool kPairedFma = BN != 128;
  static constexpr int kLdCols = 32;  // columns per double-buffered TMEM load
  // shared-memory carve-up (offsets from a 1024-byte aligned base); both CTAs
  // of a pair use identical offsets, which the pair MMA relies on
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kStages * kABytes;
  static constexpr int kOffRaw = kOffB + kStages * kBBytes;                 // prefetched x_scale [kPrefetch][256]
  static constexpr int kOffRawW = kOffRaw + kPrefetch * 256 * 4;            // prefetched w_scale [kPrefetch][256]
  static constexpr int kOffBar = kOffRawW + kPrefetch * 256 * 4;
  static constexpr int kNumBars = 2 * kStages + 2 * kTmemBufs + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;   // + alignment slack
  static_assert(kStages >= 2, "pipeline needs two stages");
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
  static_assert(kTileM * kPitch32 * 4 <= kOffRaw, "fp32 output staging must fit in the stage ring");
};

constexpr int kMaxPeers = 7;  // peer outputs of fack_gemm_bs_bcast (8 GPUs per node)
constexpr int kMaxRanks = kMaxPeers + 1;
constexpr unsigned int kStExchange = 32u;  // a peer's completion signal did not arrive in time

// Completion state of the fused all-gather, one per rank in that rank's
// device memory (FACK_XCHG_BYTES, zero before first use), mapped into every
// other rank.  done[s] is added to only by rank s (over NVLink): each CTA of
// an exchange launch on rank s adds its share of 2^32 once its stores into
// this rank's output have landed, the shares of one launch summing to exactly
// 2^32 whatever its grid size.  So done[s] >= e * 2^32 once rank s's first e
// exchanges have landed here.
struct XchgState {
  unsigned int reserved[2];
  unsigned long long seq;             // exchanges this rank has completed
  unsigned long long done[kMaxRanks];
};
constexpr int kXchgShift = 32;        // one exchange adds 2^32 to each peer's done[rank]
static_assert(sizeof(XchgState) <= FACK_XCHG_BYTES, "exchange state outgrew FACK_XCHG_BYTES");

struct Params {
  const float* x_scale;
  int64_t xs_sm, xs_sk;
  const float* w_scale;        // [N/128][K/128]
  __nv_bfloat16* out;
  int64_t ldo;
  // the same output block in other GPUs' memory (peer mappings, same ldo):
  // every bf16 result is stored to out and to each peer_out[0..n_peer)
  __nv_bfloat16* peer_out[kMaxPeers];
  int n_peer;
  // fused all-gather completion (NULL: none): this rank's state, and for each
  // peer d the slot done[rank] of that peer's state (peer mapping)
  XchgState* xchg;
  unsigned long long* peer_done[kMaxPeers];
  int rank, world;
  float* partials;             // [tiles][S][128][BN] fp32 for S > 1; NULL = reduce through DSMEM
                               // persistent kernel with a tail split: [tail pieces][128][BN] fp32
  int tail_rem;                // persistent kernel: the last tail_rem tiles of the launch order are split ...
  int tail_split;              // ... over K into tail_split pieces each (0 = no tail split)
  int M, N, K, KB;
  int split;
  int w_packed;
  uint64_t timeout_ns;
  uint64_t xchg_timeout_ns;
};

// This CTA's part of an exchange launch (one thread, after a system fence
// that covers the CTA's peer stores): add its share of 2^32 to done[rank] of
// every peer's state.  Relaxed adds: the fence before them is the release.
__device__ __forceinline__ void xchg_post(unsigned long long* const* peer_done, int n_peer, unsigned int cta,
                                          unsigned int ctas) {
  // 2^32 = ctas * q + r + 1 with q, r the quotient and remainder of 2^32 - 1
  const unsigned int q = 0xffffffffu / ctas, r = 0xffffffffu % ctas;
  const bool exact = (r + 1u == ctas);
  const unsigned long long base = static_cast<unsigned long long>(q) + (exact ? 1ull : 0ull);
  const unsigned int rem = exact ? 0u : r + 1u;
  const unsigned long long share = base + (cta < rem ? 1ull : 0ull);
  for (int d = 0; d < n_peer; ++d) red_add_relaxed_sys_u64(peer_done[d], share);
}

// The wait of one exchange step on this rank (one thread of the launch):
// until every peer's shares for this step have arrived (acquire loads of this
// rank's done[]), then count the step.  The wait is bounded: on expiry it ORs
// kStExchange into the status word and returns.  Every call on a rank's state
// comes from one stream, in the same order on every rank, so the step numbers
// agree; a peer already posting its next step only pushes done[] further.
__device__ __noinline__ void xchg_wait(XchgState* x, int rank, int world, uint64_t timeout_ns,
                                       unsigned int* status) {
  const unsigned long long seq = x->seq + 1;
  x->seq = seq;
  const unsigned long long target = seq << kXchgShift;
  const uint64_t t0 = global_timer_ns();
  for (int s = 0; s < world; ++s) {
    if (s == rank) continue;
    while (ld_acquire_sys_u64(&x->done[s]) < target) {
      if (global_timer_ns() - t0 > timeout_ns) {
        atomicOr(status, kStExchange);
        return;
      }
      __nanosleep(64);
    }
  }
}

// After a thread's peer stores.  Without the fused exchange each storing
// thread makes its stores visible system-wide itself.  With it, xchg_complete
// fences once per CTA behind a CTA barrier instead: a fence is cumulative over
// the stores that the barrier orders before it, and hundreds of per-thread
// system fences, each waiting on NVLink write acknowledgements, cost more than
// the stores they follow.
__device__ __forceinline__ void peer_store_fence(const Params& p) {
  if (p.n_peer && !p.xchg) __threadfence_system();
}

// End of a GEMM launch with peer stores (all threads of each CTA): the CTA's
// stores are made visible system-wide (barrier, then one system fence), the
// CTA posts its share to every peer straight away, and CTA 0 waits for every
// peer's shares.  No CTA waits on another CTA of its own grid (no ticket):
// the last peer store to land is followed only by one NVLink add.  The grid
// therefore completes only once every rank's blocks have landed in this
// rank's output, so no separate barrier or collective is needed on the stream.
// The posting thread's work is kept out of line so that its registers are
// allocated apart from the kernels'.
__device__ __noinline__ void xchg_post_and_wait(const Params& p, unsigned int* status) {
  const unsigned int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  __threadfence_system();
  xchg_post(p.peer_done, p.n_peer, cta, gridDim.x * gridDim.y * gridDim.z);
  if (cta == 0) xchg_wait(p.xchg, p.rank, p.world, p.xchg_timeout_ns, status);
}

__device__ __forceinline__ void xchg_complete(const Params& p, unsigned int* status) {
  __syncthreads();
  if (threadIdx.x == 0) xchg_post_and_wait(p, status);
}

__device__ __forceinline__ uint2 pack_bf16x4(const float4& v) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 pk;
  pk.x = *reinterpret_cast<uint32_t*>(&lo);
  pk.y = *reinterpret_cast<uint32_t*>(&hi);
  return pk;
}

// Element offset `off` of the output: each peer's copy first (the NVLink
// stores have the longer way to go), then this GPU's.
__device__ __forceinline__ void store_out4(const Params& p, int64_t off, uint32_t v) {
  for (int d = 0; d < p.n_peer; ++d) *reinterpret_cast<uint32_t*>(p.peer_out[d] + off) = v;
  *reinterpret_cast<uint32_t*>(p.out + off) = v;
}
__device__ __forceinline__ void store_out8(const Params& p, int64_t off, const uint2& v) {
  for (int d = 0; d < p.n_peer; ++d) *reinterpret_cast<uint2*>(p.peer_out[d] + off) = v;
  *reinterpret_cast<uint2*>(p.out + off) = v;
}
__device__ __forceinline__ void store_out16(const Params& p, int64_t off, const uint4& v) {
  for (int d = 0; d < p.n_peer; ++d) *reinterpret_cast<uint4*>(p.peer_out[d] + off) = v;
  *reinterpret_cast<uint4*>(p.out + off) = v;
}

// Split-K reduction over distributed shared memory: rows [r0, r1) of the
// tile, summed over the S cluster CTAs' staged fp32 partials in rank order.
// One remote load per slice per item in flight: the pull is bound by the
// distributed-shared-memory bandwidth, not by latency.  Kept out of line so
// its registers are allocated apart from the rescale loop.
template <int BN, int PITCH>
__device__ __noinline__ void reduce_dsmem(uint32_t stg, int S, int rank0, int rank_step, int r0, int r1,
                                          const Params& p, int64_t off0) {
  constexpr int kRowF4 = BN / 4;
  const int items = (r1 > r0 ? r1 - r0 : 0) * kRowF4;
  for (int it = threadIdx.x; it < items; it += kThreads) {
    const int r = r0 + it / kRowF4;
    const int c4 = it % kRowF4;
    const uint32_t addr = stg + static_cast<uint32_t>((r * PITCH + c4 * 4) * 4);
    float4 sum = dsmem_ld4(dsmem_map(addr, rank0));
    for (int t = 1; t < S; ++t) {
      const float4 v = dsmem_ld4(dsmem_map(addr, rank0 + t * rank_step));
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    store_out8(p, off0 + r * p.ldo + c4 * 4, pack_bf16x4(sum));
  }
}

// Copy the staged fp32 partial to its workspace slot: the valid rows other
// slices reduce (every row outside [keep0, keep1), which this CTA reduces
// from its own staging).  An SM stores at only ~24 B/clk, so nothing is
// written that no other CTA reads.
template <int BN, int PITCH>
__device__ __noinline__ void copy_partial(const float* stg, int rows, int keep0, int keep1, float* part) {
  constexpr int kRowF4 = BN / 4;
  const int kept = keep1 > keep0 ? keep1 - keep0 : 0;
  for (int c = threadIdx.x; c < (rows - kept) * kRowF4; c += kThreads) {
    int r = c / kRowF4;
    r += r >= keep0 ? kept : 0;
    const int c4 = c % kRowF4;
    __stcg(reinterpret_cast<float4*>(part + r * BN + c4 * 4),
           *reinterpret_cast<const float4*>(stg + r * PITCH + c4 * 4));
  }
}

// Split-K reduction through the workspace: rows [r0, r1), slices in order
// 0..S-1; slice `self` comes from this CTA's own staging tile (pitch PITCH),
// the others from the workspace (L2).
template <int BN, int PITCH>
__device__ __noinline__ void reduce_global(const float* part0, const float* stg, int self, int S, int r0, int r1,
                                           const Params& p, int64_t off0) {
  constexpr int kRowF4 = BN / 4;
  const int items = (r1 > r0 ? r1 - r0 : 0) * kRowF4;
  for (int it = threadIdx.x; it < items; it += kThreads) {
    const int r = r0 + it / kRowF4;
    const int c = (it % kRowF4) * 4;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < S; ++t) {
      const float4 v = t == self ? *reinterpret_cast<const float4*>(stg + r * PITCH + c)
                                 : __ldcg(reinterpret_cast<const float4*>(part0 + (static_cast<int64_t>(t) * kTileM + r) * BN + c));
      if (t == 0) {
        sum = v;
      } else {
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
    }
    store_out8(p, off0 + r * p.ldo + c, pack_bf16x4(sum));
  }
}

// TMA of one K block of a BN-row weight tile starting at weight row wr0:
// packed layout (tile (nb, kb) is 128 rows x 128 B at row (nb*KB + kb)*128)
// or row-major [N, K].
// A 224-row tile (first row a multiple of 32, not of 128) is loaded from the
// packed layout as seven 32-row boxes, each inside one packed 128-row tile
// (the host encodes 32-row boxes for it).
template <int WROWS>
__device__ __forceinline__ void load_w_tile(uint32_t dst, const CUtensorMap* map, uint32_t bar, const Params& p,
                                            int wr0, int kb, uint64_t pol) {
  if (p.w_packed) {
    if constexpr (WROWS == 224) {
#pragma unroll
      for (int j = 0; j < WROWS / 32; ++j) {
        const int r = wr0 + 32 * j;
        tma_load_2d(dst + j * 4096, map, bar, 0, ((r >> 7) * p.KB + kb) * kBlk + (r & 127), pol);
      }
    } else {
#pragma unroll
      for (int t = 0; t < (WROWS + 127) / 128; ++t)
        tma_load_2d(dst + t * 16384, map, bar, 0, (((wr0 >> 7) + t) * p.KB + kb) * kBlk + (wr0 & 127), pol);
    }
  } else {
    tma_load_2d(dst, map, bar, kb * kBlk, wr0, pol);
  }
}

// PAIR = false: one CTA per 128-token x BN-weight-row tile (cta_group::1).
// PAIR = true : two CTAs (cluster x pair) share a 256-token x BN tile through
//   tcgen05 cta_group::2: each CTA loads its own 128 tokens and half of the
//   BN weight rows, the even-ranked CTA (leader) issues the M=256 MMA, and
//   each CTA receives its 128 x BN accumulator rows in its own TMEM.  Weight
//   bytes per CTA halve; the rescale / epilogue code is the same.
template <int BN, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bs_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
               const __grid_constant__ Params p) {
  using C = Cfg<BN, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // grid: single CTAs (x = weight tile, y = token tile); pairs (x = token
  // tile, so that the pair lies along the cluster's x dimension, y = weight
  // tile); z = K slice.  The launch order is remapped (grouped rasterization):
  // within a K slice consecutive CTAs walk the token tiles of a band of
  // kGroupM tiles before moving to the next weight tile, so the CTAs resident
  // at one time share both operands in L2 instead of streaming all weights
  // once per row of token tiles.
  int mt, nt;
  {
    const int unit = PAIR ? 2 : 1;                               // CTAs per token-tile slot
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
  const int s = blockIdx.z;                        // K slice
  const int S = p.split;
  const int m0 = mt * kTileM;
  const int n0 = nt * BN;
  const int kb0 = (s * p.KB) / S;
  const int kb1 = ((s + 1) * p.KB) / S;
  const int nk = kb1 - kb0;
  const int rows = min(kTileM, p.M - m0);    // valid tokens in this tile (may be <= 0 for a pair's second CTA)
  const int quarters = rows > 0 ? (rows + 31) >> 5 : 0;   // TMEM lane quarters holding valid tokens
  // pair bookkeeping: cluster dims (2, 1, S), rank = (mt & 1) + 2 * s
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = !PAIR || (mt & 1) == 0;
  const uint32_t leader_rank = crank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader_rank);
  // rescale warps that release each TMEM buffer: this CTA's (and, in a pair,
  // the other CTA's) warps whose lane quarter holds valid tokens
  int release_warps = 2 * quarters;
  if (PAIR) {
    const int other = min(kTileM, p.M - (m0 ^ kTileM));  // the other CTA's token tile: mt ^ 1
    release_warps = 2 * ((rows > 0 ? (rows + 31) >> 5 : 0) + (other > 0 ? (other + 31) >> 5 : 0));
  }

  const uint32_t bar0 = base + C::kOffBar;
  auto bar_full = [&](int i) { return bar0 + 8u * i; };
  auto bar_empty = [&](int i) { return bar0 + 8u * (C::kStages + i); };
  auto bar_tfull = [&](int i) { return bar0 + 8u * (2 * C::kStages + i); };
  auto bar_tempty = [&](int i) { return bar0 + 8u * (2 * C::kStages + C::kTmemBufs + i); };
  const uint32_t bar_drain = bar0 + 8u * (2 * C::kStages + 2 * C::kTmemBufs);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(bar_full(i), 1);
      mbar_init(bar_empty(i), 1);
    }
    for (int i = 0; i < C::kTmemBufs; ++i) {
      mbar_init(bar_tfull(i), 1);
      mbar_init(bar_tempty(i), release_warps > 0 ? release_warps : 1);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_addr(tmem_slot), C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
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
  // Everything above touches only this CTA's own resources, so with
  // programmatic dependent launch it overlaps the previous kernel's tail;
  // nothing the previous kernel may have written is read before this wait.
  grid_dependency_wait();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t tmo = p.timeout_ns;
  unsigned int* status = &g_status;

  int produced = 0;  // TMA stages issued (producer lane only)

  if (warp < kEpiWarp0) {
    // Control warpgroup: hand registers to the two rescale warpgroups.
    regs_dec<kCtrlRegs>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer --
      if (lane == 0) {
        const uint64_t pol_w = policy_evict_first();   // weights stream once
        const uint64_t pol_x = policy_evict_last();    // tokens are re-read by every weight tile
        const int wr0 = n0 + (PAIR ? static_cast<int>(mt & 1) * C::kWRows : 0);  // first weight row loaded here
        for (int i = 0; i < nk; ++i) {
          const int st = i % C::kStages;
          const uint32_t ph = (i / C::kStages) & 1;
          if (!wait_bounded(bar_empty(st), ph ^ 1u, abort_flag, status, kStProducer, tmo)) break;
          const int kb = kb0 + i;
          const uint32_t sa = base + C::kOffA + st * C::kABytes;
          const uint32_t sb = base + C::kOffB + st * C::kBBytes;
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the leader's full barrier
            const uint32_t fb = dsmem_map(bar_full(st), leader_rank);
            if (leader) mbar_arrive_expect_tx(bar_full(st), 2 * C::kStageBytes);
            tma_load_2d_pair(sa, &tmap_x, fb, kb * kBlk, m0, pol_x);
            if (p.w_packed) {
#pragma unroll
              for (int t = 0; t < (C::kWRows + 127) / 128; ++t)
                tma_load_2d_pair(sb + t * 16384, &tmap_w, fb, 0,
                                 (((wr0 >> 7) + t) * p.KB + kb) * kBlk + (wr0 & 127), pol_w);
            } else {
              tma_load_2d_pair(sb, &tmap_w, fb, kb * kBlk, wr0, pol_w);
            }
          } else {
            mbar_arrive_expect_tx(bar_full(st), C::kStageBytes);
            tma_load_2d(sa, &tmap_x, bar_full(st), kb * kBlk, m0, pol_x);
            load_w_tile<C::kWRows>(sb, &tmap_w, bar_full(st), p, wr0, kb, pol_w);
          }
          produced = i + 1;
        }
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer --
      if (lane == 0 && leader) {
        constexpr uint32_t idesc = idesc_e4m3_f32(PAIR ? 2 * kTileM : kTileM, BN);
        for (int i = 0; i < nk; ++i) {
          const int st = i % C::kStages;
          const uint32_t ph = (i / C::kStages) & 1;
          const int buf = i % C::kTmemBufs;
          const uint32_t bph = (i / C::kTmemBufs) & 1;
          if (!wait_bounded(bar_tempty(buf), bph ^ 1u, abort_flag, status, kStMma, tmo)) break;
          if (!wait_bounded(bar_full(st), ph, abort_flag, status, kStMma, tmo)) break;
          tc_fence_after();
          const uint32_t d = tmem_base + buf * BN;
          const uint64_t da = sw128_kmajor_desc(base + C::kOffA + st * C::kABytes);
          const uint64_t db = sw128_kmajor_desc(base + C::kOffB + st * C::kBBytes);
          if constexpr (PAIR) {
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) umma_f8_pair(d, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
            umma_commit_pair_mc(bar_empty(st), pair_mask);   // frees the stage in both CTAs
            umma_commit_pair_mc(bar_tfull(buf), pair_mask);  // both CTAs' accumulators are ready
          } else {
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k)  // K = 32 e4m3 elements = 32 bytes = 2 descriptor units
              umma_f8(d, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
            umma_commit(bar_empty(st));
            umma_commit(bar_tfull(buf));
          }
        }
      }
    }
  } else {
    // -------------------------------------------------- rescale / epilogue --
    regs_inc<kEpiRegs>();
    const int q = warp & 3;                       // TMEM lane quarter this warp may access
    const int h = (warp - kEpiWarp0) >> 2;        // column half
    const int col0 = h * C::kCpw;
    const int tok = q * 32 + lane;                // token row inside the tile
    // where this warp reports a released TMEM buffer: the MMA issuer's CTA
    const uint32_t tempty_base = PAIR ? dsmem_map(bar_tempty(0), leader_rank) : bar_tempty(0);
    if (q < quarters) {
      // fp32 accumulators: two per 64-bit register where the rescale uses the
      // paired FMA (its operand form), else one float each
      constexpr int kAccN = C::kPairedFma ? C::kCpw / 2 : C::kCpw;
      using AccT = typename std::conditional<C::kPairedFma, uint64_t, float>::type;
      AccT acc[kAccN];
#pragma unroll
      for (int j = 0; j < kAccN; ++j) acc[j] = AccT(0);
      // columns j, j+1 (j even) of the accumulator
      auto acc_pair = [&](int j) -> float2 {
        if constexpr (C::kPairedFma)
          return unpack_f32x2(acc[j >> 1]);
        else
          return make_float2(acc[j], acc[j + 1]);
      };
      // Scales: x_scale[m0+tok, kb] and w_scale[block of this column half, kb]
      // prefetched kPrefetch K blocks ahead with cp.async into this thread's
      // private shared slots (one commit group per K block).
      const int et = (warp - kEpiWarp0) * 32 + lane;
      const bool has = tok < rows;
      const float* xs_row = p.x_scale + static_cast<int64_t>(has ? m0 + tok : 0) * p.xs_sm;  // row 0 exists
      const float* ws_row = p.w_scale + static_cast<int64_t>((n0 + col0) >> 7) * p.KB;
      const uint32_t raw_x = base + C::kOffRaw + et * 4;
      const uint32_t raw_w = base + C::kOffRawW + et * 4;
      const float* raw_xp = reinterpret_cast<const float*>(smem + C::kOffRaw) + et;
      const float* raw_wp = reinterpret_cast<const float*>(smem + C::kOffRawW) + et;
      auto prefetch = [&](int i) {  // copies for K block kb0 + i into slot i % kPrefetch
        if (i < nk) {
          const int off = (i % kPrefetch) * 256 * 4;
          const int kb = kb0 + i;
          cp_async4(raw_x + off, xs_row + static_cast<int64_t>(kb) * p.xs_sk, has ? 4u : 0u);
          cp_async4(raw_w + off, ws_row + kb, 4u);
        }
        cp_async_commit();  // one group per K block, empty past the end
      };
#pragma unroll
      for (int d = 0; d < kPrefetch; ++d) prefetch(d);
      bool done = true;
      for (int i = 0; i < nk; ++i) {
        const int buf = i % C::kTmemBufs;
        const uint32_t bph = (i / C::kTmemBufs) & 1;
        cp_async_wait<kPrefetch - 1>();  // this thread's copies for K block i have landed
        const float sc = raw_xp[(i % kPrefetch) * 256] * raw_wp[(i % kPrefetch) * 256];
        const uint64_t sc2 = C::kPairedFma ? pack_f32x2(sc, sc) : 0ull;
        prefetch(i + kPrefetch);
        // tcgen05.ld is .sync.aligned: the whole warp must agree before using it.
        const bool got = wait_bounded(bar_tfull(buf), bph, abort_flag, status, kStEpilogue, tmo);
        if (!__all_sync(0xffffffffu, got)) {
          done = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN + col0;
        // Double-buffered kLd-column TMEM loads: chunk c+1 is in flight while
        // chunk c is folded into the accumulators.
        constexpr int kLd = C::kLdCols;
        constexpr int kChunks = C::kCpw / kLd;
        auto ld_issue = [&](uint32_t addr, uint32_t(&v)[kLd]) {
          if constexpr (kLd == 32) tmem_ld32_nowait(addr, v); else tmem_ld16_nowait(addr, v);
        };
        auto ld_wait = [&](uint32_t(&v)[kLd]) {
          if constexpr (kLd == 32) tmem_wait32(v); else tmem_wait16(v);
        };
        auto fold = [&](int c, const uint32_t(&v)[kLd]) {
#pragma unroll
          for (int t = 0; t < kLd; t += 2) {
            if constexpr (C::kPairedFma) {
              fma2_acc(acc[(c * kLd + t) >> 1], v[t], v[t + 1], sc2);
            } else {
              acc[c * kLd + t] = fmaf(__uint_as_float(v[t]), sc, acc[c * kLd + t]);
              acc[c * kLd + t + 1] = fmaf(__uint_as_float(v[t + 1]), sc, acc[c * kLd + t + 1]);
            }
          }
        };
        uint32_t va[kLd], vb[kLd];
        ld_issue(taddr, va);
        ld_wait(va);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          if ((c & 1) == 0) {
            if (c + 1 < kChunks) ld_issue(taddr + (c + 1) * kLd, vb);
            fold(c, va);
            if (c + 1 < kChunks) ld_wait(vb);
          } else {
            if (c + 1 < kChunks) ld_issue(taddr + (c + 1) * kLd, va);
            fold(c, vb);
            if (c + 1 < kChunks) ld_wait(va);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_remote(tempty_base + 8u * buf);
          else
            mbar_arrive(bar_tempty(buf));
        }
      }
      cp_async_wait<0>();  // no copy may land after the CTA exits
      if (done && *abort_flag == 0) {
        // Stage this thread's row segment in the idle stage ring (every TMA
        // copy was consumed and the last MMA reading it completed before this
        // warp's final wait); the padded pitch spreads rows over banks.
        if (S > 1) {
          float* row = reinterpret_cast<float*>(smem + C::kOffA) + tok * C::kPitch32 + col0;
#pragma unroll
          for (int j = 0; j < C::kCpw; j += 4) {
            const float2 lo = acc_pair(j), hi = acc_pair(j + 2);
            *reinterpret_cast<float4*>(row + j) = make_float4(lo.x, lo.y, hi.x, hi.y);
          }
        } else {
          __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffA) + tok * C::kPitch16 + col0;
#pragma unroll
          for (int j = 0; j < C::kCpw; j += 8) {
            uint4 v;
            const float2 f0 = acc_pair(j), f1 = acc_pair(j + 2);
            const float2 f2 = acc_pair(j + 4), f3 = acc_pair(j + 6);
            __nv_bfloat162 b0 = __floats2bfloat162_rn(f0.x, f0.y);
            __nv_bfloat162 b1 = __floats2bfloat162_rn(f1.x, f1.y);
            __nv_bfloat162 b2 = __floats2bfloat162_rn(f2.x, f2.y);
            __nv_bfloat162 b3 = __floats2bfloat162_rn(f3.x, f3.y);
            v.x = *reinterpret_cast<uint32_t*>(&b0);
            v.y = *reinterpret_cast<uint32_t*>(&b1);
            v.z = *reinterpret_cast<uint32_t*>(&b2);
            v.w = *reinterpret_cast<uint32_t*>(&b3);
            *reinterpret_cast<uint4*>(row + j) = v;
          }
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown --
  // The next launch may start its prologue now; it still waits for this whole
  // grid to finish before reading anything (grid_dependency_wait).
  grid_launch_dependents();
  __syncwarp();  // lane 0 of the producer and MMA warps rejoins the other lanes
  tc_fence_before();
  __syncthreads();  // every role of this CTA has left its loop
  tc_fence_after();
  if (warp == 0) {
    // Producer: if the pipeline was abandoned, wait (bounded, fresh deadline)
    // for the TMA copies it issued so none lands after the CTA has exited.
    if (*abort_flag && lane == 0) {
      const int first = produced > C::kStages ? produced - C::kStages : 0;
      volatile int no_abort = 0;
      if (leader) {
        for (int i = first; i < produced; ++i)
          wait_bounded(bar_full(i % C::kStages), (i / C::kStages) & 1, &no_abort, status, kStDrain, tmo);
      } else {
        // a pair's second CTA signals its loads on the leader's barrier and
        // cannot observe them: give them a bounded 50 us to land
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 50000u) __nanosleep(1000);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // No MMA may still be writing TMEM when it is freed: commit arrives once
    // every earlier tcgen05.mma of this thread has completed.
    if (lane == 0 && leader) {
      if constexpr (PAIR)
        umma_commit_pair(bar_drain);
      else
        umma_commit(bar_drain);
      volatile int no_abort = 0;
      wait_bounded(bar_drain, 0, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
  }
  if constexpr (PAIR) {
    // the leader's MMAs have drained and the peer's loads were consumed (or
    // drained): only now may either CTA free its TMEM, and neither exits
    // while the other may still signal its barriers
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
  }
  const bool ok = (*abort_flag == 0);
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else
      tmem_dealloc(tmem_base, C::kTmemCols);
  }

  // Output stores; every path returns here so that, with the fused
  // all-gather, every CTA reaches the completion step below.
  auto store_output = [&]() {
    if (S == 1) {
      if (!ok || rows <= 0) return;
      // 16-byte vectors of the staged bf16 tile along rows of Y
      const __nv_bfloat16* stg = reinterpret_cast<const __nv_bfloat16*>(smem + C::kOffA);
      constexpr int kRowChunks = BN / 8;
      for (int c = threadIdx.x; c < rows * kRowChunks; c += kThreads) {
        const int r = c / kRowChunks, cc = c % kRowChunks;
        const uint4 v = *reinterpret_cast<const uint4*>(stg + r * C::kPitch16 + cc * 8);
        store_out16(p, static_cast<int64_t>(m0 + r) * p.ldo + n0 + cc * 8, v);
      }
      peer_store_fence(p);
      return;
    }

    // Split-K.  Every CTA of the cluster arrives at every cluster barrier, also
    // after an abort, so none waits forever; each then sums a disjoint block of
    // rows over the slices in fixed order 0..S-1 (bitwise reproducible).
    const int rows_v = rows > 0 ? rows : 0;
    const int per = (rows_v + S - 1) / S;
    const int r0 = s * per;
    const int r1 = min(rows_v, r0 + per);
    const int rank_step = PAIR ? 2 : 1;               // cluster rank of slice t: (mt & 1) + rank_step * t
    const int rank0 = PAIR ? static_cast<int>(mt & 1) : 0;
    if (p.partials == nullptr) {
      // Partials stay in each CTA's shared staging tile; peers read them over
      // distributed shared memory.  The second barrier keeps every CTA (and so
      // its shared memory) alive until all peers have finished reading.
      cluster_sync_all();
      if (ok)
        reduce_dsmem<BN, C::kPitch32>(base + C::kOffA, S, rank0, rank_step, r0, r1, p,
                                      static_cast<int64_t>(m0) * p.ldo + n0);
      peer_store_fence(p);
      cluster_sync_all();
      return;
    }
    // Caller-provided workspace (reduce-scatter through L2): each slice writes
    // the rows the other slices reduce, the cluster barrier publishes them, and
    // each slice sums its own rows from the workspace and its own staging.  No
    // CTA reads another's shared memory, so there is no second barrier.
    const int64_t tile = static_cast<int64_t>(mt) * (p.N / BN) + nt;
    const float* stg32 = reinterpret_cast<const float*>(smem + C::kOffA);
    if (ok) {
      copy_partial<BN, C::kPitch32>(stg32, rows_v, r0, r1, p.partials + (tile * S + s) * kTileM * BN);
      __threadfence();
    }
    cluster_sync_all();
    if (!ok) return;
    reduce_global<BN, C::kPitch32>(p.partials + tile * S * kTileM * BN, stg32, s, S, r0, r1, p,
                                   static_cast<int64_t>(m0) * p.ldo + n0);
    peer_store_fence(p);
  };
  store_output();
  if (p.xchg) xchg_complete(p, status);
}

// ------------------------------------------------- persistent (multi-wave) --
// Unsplit plans whose tiles outnumber the SMs (the prefill layer: 1792 tiles of
// 128 x 256) run persistently: one CTA per SM walks its tiles (every
// gridDim.x-th tile of the grouped launch order, so the tiles in flight at one
// time still share operands in L2), and
//  * the TMA producer and the MMA issuer run one continuous pipeline over all
//    of the CTA's tiles and K blocks, so a tile's first loads and MMAs overlap
//    the previous tile's last rescale and its epilogue;
//  * the rescale warps hand each finished bf16 tile to a staging buffer of its
//    own and go on with the next tile; two store warps (warps 2-3, idle in the
//    one-tile kernel) copy it to Y -- and, for the fused all-gather, to every
//    peer's Y over NVLink -- while the next tile computes;
//  * barrier set-up, TMEM allocation and teardown happen once per SM, not
//    once per tile.
// The per-tile arithmetic (scales, paired FMA, bf16 rounding) is the one-tile
// kernel's, so results are bitwise identical to it.
constexpr int kPersistSmem = 232448 - 1024 - 256;   // dynamic budget minus alignment slack and misc

template <int BN>
struct PCfg {
  static constexpr int kABytes = kTileM * kBlk;             // 16 KB token tile
  static constexpr int kBBytes = BN * kBlk;                 // weight tile
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kPitch16 = BN + 8;                   // bf16 staging pitch (elements)
  static constexpr int kStgBytes = kTileM * kPitch16 * 2;   // one staged output tile
  // two staging buffers where shared memory allows (weight tiles up to 128):
  // the store warps then drain tile i while tile i + 1 is staged
  static constexpr int kStgBufs = BN <= 128 ? 2 : 1;
  // w_scale values per thread and K block: a 224-row tile's half (112 rows)
  // may span two 128-row scale blocks
  static constexpr int kWScales = BN == 224 ? 2 : 1;
  static constexpr int kRawBytes = (1 + kWScales) * kPrefetch * 256 * 4; // prefetched x_scale and w_scale slots
  static constexpr int kFit = (kPersistSmem - kStgBufs * kStgBytes - kRawBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kTmemBufs = (512 / BN) > 4 ? 4 : (512 / BN);
  // the allocation is a power of two: 2 x 224 columns take 512
  static constexpr int kTmemCols = kTmemBufs * BN <= 256 ? 256 : 512;
  static constexpr int kCpw = BN / 2;                       // columns per rescale warp
  static constexpr bool kPairedFma = BN != 128;             // as in Cfg: the 128 tile keeps scalar FMAs
  // columns per double-buffered TMEM load: 16 for the 256 and 224 tiles,
  // whose 128 / 112 accumulator columns per thread leave no room for two
  // 32-column buffers next to the tile loop's own state
  static constexpr int kLdCols = BN >= 224 ? 16 : 32;

  static constexpr int kOffA = 0;
  static constexpr int kOffB = kStages * kABytes;
  static constexpr int kOffStg = kOffB + kStages * kBBytes;
  static constexpr int kOffRaw = kOffStg + kStgBufs * kStgBytes;
  static constexpr int kOffRawW = kOffRaw + kPrefetch * 256 * 4;
  static constexpr int kOffRawW2 = kOffRawW + kPrefetch * 256 * 4;   // second w_scale (224 tile only)
  static constexpr int kOffBar = kOffRawW + kWScales * kPrefetch * 256 * 4;
  static constexpr int kNumBars = 2 * kStages + 2 * kTmemBufs + 2 * kStgBufs + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;
  static_assert(kStages >= 3, "persistent pipeline needs three stages");
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
};

constexpr int kStoreWarp0 = 2;   // warps 2-3: store warps of the persistent kernel
constexpr int kStoreThreads = 64;

// Tile `lin` of the grouped launch order (bands of kGroupM token tiles,
// weight tiles outer within a band), as the one-tile kernel's remap.
__device__ __forceinline__ void grouped_tile(int lin, int n_tiles, int m_tiles, int& mt, int& nt) {
  const int per_group = kGroupM * n_tiles;
  const int g = lin / per_group;
  const int first = g * kGroupM;
  const int gm = min(kGroupM, m_tiles - first);
  const int r = lin - g * per_group;
  nt = r / gm;
  mt = first + r % gm;
}

// Work items of a persistent CTA: its full tiles (every gridDim.x-th tile of
// the launch order), then, with a tail split, at most one piece -- one of
// tail_split K slices of one of the last tail_rem tiles, whose fp32 partial
// goes to the workspace for tail_fixup_kernel.  Without a tail split the
// last round may leave most SMs idle (1792 = 12 x 148 + 16 prefill tiles);
// with it those tiles' K blocks are spread over the idle CTAs.
struct PWork {
  int n_tiles, m_tiles, total, KB, n_dp, piece, my_items;
  __device__ PWork(const Params& p, int BN) {
    n_tiles = p.N / BN;
    m_tiles = (p.M + kTileM - 1) / kTileM;
    total = n_tiles * m_tiles;
    KB = p.KB;
    const int b = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
    if (p.tail_split) {
      n_dp = (total - p.tail_rem) / G;  // the tiles before the tail are exactly n_dp rounds
      piece = b < p.tail_rem * p.tail_split ? b : -1;
    } else {
      n_dp = total > b ? (total - 1 - b) / G + 1 : 0;
      piece = -1;
    }
    my_items = n_dp + (piece >= 0 ? 1 : 0);
  }
  // tile and K-block range of item i
  __device__ void item(const Params& p, int i, int& mt, int& nt, int& kb0, int& kb1) const {
    if (i < n_dp) {
      grouped_tile(static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x), n_tiles, m_tiles, mt, nt);
      kb0 = 0;
      kb1 = KB;
    } else {
      const int S = p.tail_split;
      grouped_tile(total - p.tail_rem + piece / S, n_tiles, m_tiles, mt, nt);
      const int sl = piece % S;
      kb0 = (sl * KB) / S;
      kb1 = ((sl + 1) * KB) / S;
    }
  }
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bs_persistent_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                          const __grid_constant__ Params p) {
  using C = PCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const PWork w(p, BN);

  const uint32_t bar0 = base + C::kOffBar;
  auto bar_full = [&](int i) { return bar0 + 8u * i; };
  auto bar_empty = [&](int i) { return bar0 + 8u * (C::kStages + i); };
  auto bar_tfull = [&](int i) { return bar0 + 8u * (2 * C::kStages + i); };
  auto bar_tempty = [&](int i) { return bar0 + 8u * (2 * C::kStages + C::kTmemBufs + i); };
  // staging buffer b: full (staged by the rescale warps), empty (drained)
  auto bar_sfull = [&](int b) { return bar0 + 8u * (2 * C::kStages + 2 * C::kTmemBufs + b); };
  auto bar_sempty = [&](int b) { return bar0 + 8u * (2 * C::kStages + 2 * C::kTmemBufs + C::kStgBufs + b); };
  const uint32_t bar_drain = bar0 + 8u * (2 * C::kStages + 2 * C::kTmemBufs + 2 * C::kStgBufs);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(bar_full(i), 1);
      mbar_init(bar_empty(i), 1);
    }
    for (int i = 0; i < C::kTmemBufs; ++i) {
      mbar_init(bar_tfull(i), 1);
      mbar_init(bar_tempty(i), 8);          // every rescale warp releases every buffer
    }
    for (int b = 0; b < C::kStgBufs; ++b) {
      mbar_init(bar_sfull(b), 8);           // the rescale warps have staged a tile
      mbar_init(bar_sempty(b), 2);          // the store warps' copies have read it
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t tmo = p.timeout_ns;
  unsigned int* status = &g_status;
  int produced = 0;

  if (warp < kEpiWarp0) {
    regs_dec<kCtrlRegs>();
    if (warp == 0) {
      // ------------------------------------------------------------ producer --
      if (lane == 0) {
        const uint64_t pol_w = policy_evict_first();
        const uint64_t pol_x = policy_evict_last();
        int g = 0;
        bool go = true;
        for (int i = 0; i < w.my_items && go; ++i) {
          int mt, nt, kb0, kb1;
          w.item(p, i, mt, nt, kb0, kb1);
          const int m0 = mt * kTileM, n0 = nt * BN;
          for (int kb = kb0; kb < kb1; ++kb, ++g) {
            const int st = g % C::kStages;
            const uint32_t ph = (g / C::kStages) & 1;
            if (!wait_bounded(bar_empty(st), ph ^ 1u, abort_flag, status, kStProducer, tmo)) {
              go = false;
              break;
            }
            const uint32_t sa = base + C::kOffA + st * C::kABytes;
            const uint32_t sb = base + C::kOffB + st * C::kBBytes;
            mbar_arrive_expect_tx(bar_full(st), C::kStageBytes);
            tma_load_2d(sa, &tmap_x, bar_full(st), kb * kBlk, m0, pol_x);
            load_w_tile<BN>(sb, &tmap_w, bar_full(st), p, n0, kb, pol_w);
            produced = g + 1;
          }
        }
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------- MMA issuer --
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(kTileM, BN);
        int n = w.n_dp * w.KB;
        if (w.piece >= 0) {
          int mt, nt, kb0, kb1;
          w.item(p, w.n_dp, mt, nt, kb0, kb1);
          n += kb1 - kb0;
        }
        for (int g = 0; g < n; ++g) {
          const int st = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          const int buf = g % C::kTmemBufs;
          const uint32_t bph = (g / C::kTmemBufs) & 1;
          if (!wait_bounded(bar_tempty(buf), bph ^ 1u, abort_flag, status, kStMma, tmo)) break;
          if (!wait_bounded(bar_full(st), ph, abort_flag, status, kStMma, tmo)) break;
          tc_fence_after();
          const uint32_t d = tmem_base + buf * BN;
          const uint64_t da = sw128_kmajor_desc(base + C::kOffA + st * C::kABytes);
          const uint64_t db = sw128_kmajor_desc(base + C::kOffB + st * C::kBBytes);
#pragma unroll
          for (int k = 0; k < kBlk / 32; ++k) umma_f8(d, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
          umma_commit(bar_empty(st));
          umma_commit(bar_tfull(buf));
        }
      }
    } else {
      // ---------------------------------------------------------- store warps --
      // Each staged row (BN bf16, contiguous in Y) goes to Y and to every peer's
      // Y as one bulk copy by the TMA engine, so many rows per destination are
      // in flight at once (16-byte stores from two warps kept too few in
      // flight to feed NVLink at 8 GPUs).  The staging buffer is handed back
      // once the copies have read it.
      const int t = threadIdx.x - kStoreWarp0 * 32;   // 0..63
      constexpr uint32_t kRowBytes = BN * 2;
      constexpr int B = C::kStgBufs;
      for (int i = 0; i < w.n_dp; ++i) {
        const bool got = wait_bounded(bar_sfull(i % B), (i / B) & 1, abort_flag, status, kStEpilogue, tmo);
        if (!__all_sync(0xffffffffu, got)) break;
        int mt, nt, kb0, kb1;
        w.item(p, i, mt, nt, kb0, kb1);
        const int m0 = mt * kTileM, n0 = nt * BN;
        const int rows = min(kTileM, p.M - m0);
        const uint32_t stg = base + C::kOffStg + (i % B) * C::kStgBytes;
        for (int r = t; r < rows; r += kStoreThreads) {
          const uint32_t src = stg + static_cast<uint32_t>(r * C::kPitch16 * 2);
          const int64_t off = static_cast<int64_t>(m0 + r) * p.ldo + n0;
          for (int d = 0; d < p.n_peer; ++d) bulk_store_s2g(p.peer_out[d] + off, src, kRowBytes);
          bulk_store_s2g(p.out + off, src, kRowBytes);
        }
        bulk_commit();
        if constexpr (B == 1) {
          bulk_wait_read_all();  // the staging buffer may be overwritten
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_sempty(0));
        } else if (i >= 1) {
          // tile i's copies are queued; hand back the previous tile's buffer
          // once its copies have read it
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_sempty((i - 1) % B));
        }
      }
      bulk_wait_all();            // every row has landed in Y and the peers' Y ...
      fence_proxy_async_global();  // ... before this thread's later fences and stores
      if (p.n_peer) __threadfence_system();
    }
  } else {
    // -------------------------------------------------- rescale / epilogue --
    regs_inc<kEpiRegs>();
    const int q = warp & 3;
    const int h = (warp - kEpiWarp0) >> 2;
    const int col0 = h * C::kCpw;
    const int tok = q * 32 + lane;
    constexpr int kAccN = C::kPairedFma ? C::kCpw / 2 : C::kCpw;
    using AccT = typename std::conditional<C::kPairedFma, uint64_t, float>::type;
    AccT acc[kAccN];
    auto acc_pair = [&](int j) -> float2 {
      if constexpr (C::kPairedFma)
        return unpack_f32x2(acc[j >> 1]);
      else
        return make_float2(acc[j], acc[j + 1]);
    };
    const int et = (warp - kEpiWarp0) * 32 + lane;
    const uint32_t raw_x = base + C::kOffRaw + et * 4;
    const uint32_t raw_w = base + C::kOffRawW + et * 4;
    const uint32_t raw_w2 = base + C::kOffRawW2 + et * 4;
    const float* raw_xp = reinterpret_cast<const float*>(smem + C::kOffRaw) + et;
    const float* raw_wp = reinterpret_cast<const float*>(smem + C::kOffRawW) + et;
    const float* raw_w2p = reinterpret_cast<const float*>(smem + C::kOffRawW2) + et;
    // Scale prefetch: a cursor (item pi of this CTA, K block pkb of its range
    // [pkb0, pkb1)) that runs kPrefetch K blocks ahead of the rescale; an
    // item's scale rows are looked up once, and the flattened K block index
    // pj picks the slot.  pws2: the scale block of this thread's last column
    // (the 224 tile's halves can span two blocks).
    int pi = 0, pkb = 0, pkb1 = 0, pj = 0;
    bool phas = false;
    const float* pxs = p.x_scale;
    const float* pws = p.w_scale;
    const float* pws2 = p.w_scale;
    auto prefetch_item = [&]() {
      if (pi < w.my_items) {
        int mt, nt, kb0, kb1;
        w.item(p, pi, mt, nt, kb0, kb1);
        const int m = mt * kTileM + tok;
        phas = m < p.M;
        pxs = p.x_scale + static_cast<int64_t>(phas ? m : 0) * p.xs_sm;  // row 0 exists
        pws = p.w_scale + static_cast<int64_t>((nt * BN + col0) >> 7) * w.KB;
        pws2 = p.w_scale + static_cast<int64_t>((nt * BN + col0 + C::kCpw - 1) >> 7) * w.KB;
        pkb = kb0;
        pkb1 = kb1;
      }
    };
    auto prefetch = [&]() {
      if (pi < w.my_items) {
        const int off = (pj % kPrefetch) * 256 * 4;
        cp_async4(raw_x + off, pxs + static_cast<int64_t>(pkb) * p.xs_sk, phas ? 4u : 0u);
        cp_async4(raw_w + off, pws + pkb, 4u);
        if constexpr (C::kWScales == 2) cp_async4(raw_w2 + off, pws2 + pkb, 4u);
        if (++pkb == pkb1) {
          ++pi;
          prefetch_item();
        }
      }
      ++pj;
      cp_async_commit();  // one group per K block, empty past the end
    };
    prefetch_item();
#pragma unroll
    for (int d = 0; d < kPrefetch; ++d) prefetch();
    int g = 0;
    bool done = true;
    for (int i = 0; i < w.my_items && done; ++i) {
      int mt, nt, kb0, kb1;
      w.item(p, i, mt, nt, kb0, kb1);
      // columns of this thread's half before the next 128-row scale block
      // (only the 224 tile's halves cross one: chunks from there on take the
      // second scale)
      const int cross = C::kWScales == 2 ? 128 - ((nt * BN + col0) & 127) : C::kCpw;
#pragma unroll
      for (int j = 0; j < kAccN; ++j) acc[j] = AccT(0);
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const int buf = g % C::kTmemBufs;
        const uint32_t bph = (g / C::kTmemBufs) & 1;
        cp_async_wait<kPrefetch - 1>();
        const float xsc = raw_xp[(g % kPrefetch) * 256];
        const float sc = xsc * raw_wp[(g % kPrefetch) * 256];
        const float sc_hi = C::kWScales == 2 ? xsc * raw_w2p[(g % kPrefetch) * 256] : sc;
        const uint64_t sc2 = C::kPairedFma ? pack_f32x2(sc, sc) : 0ull;
        const uint64_t sc2_hi = C::kPairedFma ? pack_f32x2(sc_hi, sc_hi) : 0ull;
        prefetch();
        const bool got = wait_bounded(bar_tfull(buf), bph, abort_flag, status, kStEpilogue, tmo);
        if (!__all_sync(0xffffffffu, got)) {
          done = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN + col0;
        constexpr int kLd = C::kLdCols;
        constexpr int kChunks = C::kCpw / kLd;
        auto fold = [&](int c, const uint32_t(&v)[kLd]) {
          const bool hi = c * kLd >= cross;
#pragma unroll
          for (int t = 0; t < kLd; t += 2) {
            if constexpr (C::kPairedFma) {
              fma2_acc(acc[(c * kLd + t) >> 1], v[t], v[t + 1], hi ? sc2_hi : sc2);
            } else {
              acc[c * kLd + t] = fmaf(__uint_as_float(v[t]), sc, acc[c * kLd + t]);
              acc[c * kLd + t + 1] = fmaf(__uint_as_float(v[t + 1]), sc, acc[c * kLd + t + 1]);
            }
          }
        };
        auto ld_issue = [&](uint32_t addr, uint32_t(&v)[kLd]) {
          if constexpr (kLd == 32) tmem_ld32_nowait(addr, v); else tmem_ld16_nowait(addr, v);
        };
        auto ld_wait = [&](uint32_t(&v)[kLd]) {
          if constexpr (kLd == 32) tmem_wait32(v); else tmem_wait16(v);
        };
        uint32_t va[kLd], vb[kLd];
        ld_issue(taddr, va);
        ld_wait(va);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          if ((c & 1) == 0) {
            if (c + 1 < kChunks) ld_issue(taddr + (c + 1) * kLd, vb);
            fold(c, va);
            if (c + 1 < kChunks) ld_wait(vb);
          } else {
            if (c + 1 < kChunks) ld_issue(taddr + (c + 1) * kLd, va);
            fold(c, vb);
            if (c + 1 < kChunks) ld_wait(va);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_tempty(buf));
      }
      if (!done) break;
      if (i >= w.n_dp) {
        // a tail piece: this row's fp32 partial to the workspace, slot `piece`
        if (mt * kTileM + tok < p.M) {
          float* dst = p.partials + (static_cast<int64_t>(w.piece) * kTileM + tok) * BN + col0;
#pragma unroll
          for (int j = 0; j < C::kCpw; j += 4) {
            const float2 lo = acc_pair(j), hi = acc_pair(j + 2);
            __stcg(reinterpret_cast<float4*>(dst + j), make_float4(lo.x, lo.y, hi.x, hi.y));
          }
        }
        continue;
      }
      // hand the tile to the store warps once they have drained this buffer
      constexpr int B = C::kStgBufs;
      const bool free_stg = wait_bounded(bar_sempty(i % B), ((i / B) & 1) ^ 1, abort_flag, status, kStEpilogue, tmo);
      if (!__all_sync(0xffffffffu, free_stg)) {
        done = false;
        break;
      }
      __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffStg + (i % B) * C::kStgBytes) +
                           tok * C::kPitch16 + col0;
#pragma unroll
      for (int j = 0; j < C::kCpw; j += 8) {
        uint4 v;
        const float2 f0 = acc_pair(j), f1 = acc_pair(j + 2);
        const float2 f2 = acc_pair(j + 4), f3 = acc_pair(j + 6);
        __nv_bfloat162 b0 = __floats2bfloat162_rn(f0.x, f0.y);
        __nv_bfloat162 b1 = __floats2bfloat162_rn(f1.x, f1.y);
        __nv_bfloat162 b2 = __floats2bfloat162_rn(f2.x, f2.y);
        __nv_bfloat162 b3 = __floats2bfloat162_rn(f3.x, f3.y);
        v.x = *reinterpret_cast<uint32_t*>(&b0);
        v.y = *reinterpret_cast<uint32_t*>(&b1);
        v.z = *reinterpret_cast<uint32_t*>(&b2);
        v.w = *reinterpret_cast<uint32_t*>(&b3);
        *reinterpret_cast<uint4*>(row + j) = v;
      }
      fence_proxy_async_smem();  // the staged row is read by the TMA engine (bulk copies)
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfull(i % B));
    }
    cp_async_wait<0>();  // no copy may land after the CTA exits
  }

  // ------------------------------------------------------------ teardown --
  grid_launch_dependents();
  __syncwarp();
  tc_fence_before();
  __syncthreads();  // every role has left its loop; the store warps have drained every staged tile
  tc_fence_after();
  if (warp == 0) {
    if (*abort_flag && lane == 0) {
      const int first = produced > C::kStages ? produced - C::kStages : 0;
      volatile int no_abort = 0;
      for (int i = first; i < produced; ++i)
        wait_bounded(bar_full(i % C::kStages), (i / C::kStages) & 1, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      umma_commit(bar_drain);
      volatile int no_abort = 0;
      wait_bounded(bar_drain, 0, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (p.xchg) xchg_complete(p, status);
}

// The tail tiles of a persistent launch with a tail split: CTA
// (tail tile t, row chunk c) sums the tail_split fp32 partials of rows
// [c*rows_per, (c+1)*rows_per) of tile t in slice order 0..S-1 (bitwise
// reproducible) and stores bf16 to Y (and the peers' Y).  Launched right after
// the persistent kernel in the same stream (a plain launch: its wait for the
// persistent grid is a no-op); with the fused all-gather it runs the
// completion step.
constexpr int kFixupThreads = 256;
constexpr int kMaxTailSplit = 8;   // K slices per tail tile at most

template <int BN>
__global__ void __launch_bounds__(kFixupThreads)
gemm_bs_tail_fixup_kernel(const __grid_constant__ Params p, int chunks) {
  grid_dependency_wait();
  const int n_tiles = p.N / BN;
  const int m_tiles = (p.M + kTileM - 1) / kTileM;
  const int total = n_tiles * m_tiles;
  const int t = static_cast<int>(blockIdx.x) / chunks;
  const int c = static_cast<int>(blockIdx.x) % chunks;
  int mt, nt;
  grouped_tile(total - p.tail_rem + t, n_tiles, m_tiles, mt, nt);
  const int m0 = mt * kTileM, n0 = nt * BN;
  const int rows = min(kTileM, p.M - m0);
  const int rows_per = (kTileM + chunks - 1) / chunks;
  const int r0 = c * rows_per, r1 = min(rows, r0 + rows_per);
  const int S = p.tail_split;
  const float* part0 = p.partials + static_cast<int64_t>(t) * S * kTileM * BN;
  constexpr int kRowF4 = BN / 4;
  const int items = (r1 > r0 ? r1 - r0 : 0) * kRowF4;
  for (int it = threadIdx.x; it < items; it += kFixupThreads) {
    const int r = r0 + it / kRowF4;
    const int cc = (it % kRowF4) * 4;
    // every slice's load in flight at once, then the sum in slice order
    float4 v[kMaxTailSplit];
#pragma unroll
    for (int sl = 0; sl < kMaxTailSplit; ++sl)
      if (sl < S) v[sl] = __ldcg(reinterpret_cast<const float4*>(part0 + (static_cast<int64_t>(sl) * kTileM + r) * BN + cc));
    float4 sum = v[0];
#pragma unroll
    for (int sl = 1; sl < kMaxTailSplit; ++sl) {
      if (sl < S) {
        sum.x += v[sl].x;
        sum.y += v[sl].y;
        sum.z += v[sl].z;
        sum.w += v[sl].w;
      }
    }
    store_out8(p, static_cast<int64_t>(m0 + r) * p.ldo + n0 + cc, pack_bf16x4(sum));
  }
  peer_store_fence(p);
  grid_launch_dependents();
  if (p.xchg) xchg_complete(p, &g_status);
}

// ------------------------------------------------------ small-M (swapped) --
// For M <= 64 tokens the operands swap sides: a CTA owns 128 weight rows
// (the UMMA M side, TMEM lanes) x MT tokens (the N side, MT = 16/32/64 TMEM
// columns).  Every weight byte is then read once per K slice instead of once
// per 128-token tile row, each TMEM accumulator is only MT columns wide -- 8
// of them keep the MMA up to 8 K blocks ahead of the rescale -- and a K
// slice's partial is 128 x MT fp32 (8-32 KB), so the split-K exchange is
// small.  Per K block the scale of weight row n and token t is
// w_scale[n0/128, kb] (one value per tile) * x_scale[t, kb]; all of them are
// prefetched into shared memory when the CTA starts.
template <int MT>
struct SwapCfg {
  static_assert(MT == 16 || MT == 32 || MT == 64, "token tile must be 16, 32 or 64");
  static constexpr int kThreads = 192;               // warp 0 TMA, warp 1 MMA, warps 2-5 rescale
  static constexpr int kWBytes = 128 * kBlk;         // 16 KB weight tile (UMMA A)
  static constexpr int kXBytes = MT * kBlk;          // token tile (UMMA B)
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kStages = 6;
  static constexpr int kBufs = 8;                    // TMEM accumulators of MT columns
  static constexpr int kTmemCols = kBufs * MT;       // 128, 256, 512
  static constexpr int kMaxKb = kSwapMaxKb;          // K blocks per CTA whose scales are prefetched
  static constexpr int kPitch = 128 + 4;             // fp32 staging: one row of 128 weight rows per token
  static constexpr int kOffW = 0;
  static constexpr int kOffX = kStages * kWBytes;
  static constexpr int kOffXs = kOffX + kStages * kXBytes;   // x_scale [kMaxKb][MT]
  static constexpr int kOffWs = kOffXs + kMaxKb * MT * 4;    // w_scale [kMaxKb]
  static constexpr int kOffBar = kOffWs + kMaxKb * 4;
  static constexpr int kNumBars = 2 * kStages + 2 * kBufs + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;
  static_assert(MT * kPitch * 4 <= kOffXs, "staging must fit in the stage ring");
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
};

template <int MT>
__global__ void __launch_bounds__(SwapCfg<MT>::kThreads, 1)
gemm_bs_swap_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ Params p) {
  using C = SwapCfg<MT>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int nt = blockIdx.x;                       // 128-row weight tile
  const int s = blockIdx.z;                        // K slice
  const int S = p.split;
  const int n0 = nt * 128;
  const int kb0 = (s * p.KB) / S;
  const int nk = ((s + 1) * p.KB) / S - kb0;       // <= kMaxKb (checked on the host)
  const int M = p.M;                               // <= MT

  const uint32_t bar0 = base + C::kOffBar;
  auto bar_full = [&](int i) { return bar0 + 8u * i; };
  auto bar_empty = [&](int i) { return bar0 + 8u * (C::kStages + i); };
  auto bar_tfull = [&](int i) { return bar0 + 8u * (2 * C::kStages + i); };
  auto bar_tempty = [&](int i) { return bar0 + 8u * (2 * C::kStages + C::kBufs + i); };
  const uint32_t bar_drain = bar0 + 8u * (2 * C::kStages + 2 * C::kBufs);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);
  float* xs_s = reinterpret_cast<float*>(smem + C::kOffXs);
  float* ws_s = reinterpret_cast<float*>(smem + C::kOffWs);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(bar_full(i), 1);
      mbar_init(bar_empty(i), 1);
    }
    for (int i = 0; i < C::kBufs; ++i) {
      mbar_init(bar_tfull(i), 1);
      mbar_init(bar_tempty(i), 4);             // one arrival per rescale warp
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t tmo = p.timeout_ns;
  unsigned int* status = &g_status;
  int produced = 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        if (!wait_bounded(bar_empty(st), ph ^ 1u, abort_flag, status, kStProducer, tmo)) break;
        const int kb = kb0 + i;
        const uint32_t sw = base + C::kOffW + st * C::kWBytes;
        const uint32_t sx = base + C::kOffX + st * C::kXBytes;
        mbar_arrive_expect_tx(bar_full(st), C::kStageBytes);
        if (p.w_packed)
          tma_load_2d(sw, &tmap_w, bar_full(st), 0, (nt * p.KB + kb) * kBlk, pol_w);
        else
          tma_load_2d(sw, &tmap_w, bar_full(st), kb * kBlk, n0, pol_w);
        tma_load_2d(sx, &tmap_x, bar_full(st), kb * kBlk, 0, pol_x);   // rows >= M read as zero
        produced = i + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, MT);
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        const int buf = i % C::kBufs;
        const uint32_t bph = (i / C::kBufs) & 1;
        if (!wait_bounded(bar_tempty(buf), bph ^ 1u, abort_flag, status, kStMma, tmo)) break;
        if (!wait_bounded(bar_full(st), ph, abort_flag, status, kStMma, tmo)) break;
        tc_fence_after();
        const uint64_t da = sw128_kmajor_desc(base + C::kOffW + st * C::kWBytes);
        const uint64_t db = sw128_kmajor_desc(base + C::kOffX + st * C::kXBytes);
#pragma unroll
        for (int k = 0; k < kBlk / 32; ++k) umma_f8(tmem_base + buf * MT, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
        umma_commit(bar_empty(st));
        umma_commit(bar_tfull(buf));
      }
    }
  } else {
    // ------------------------------------------------------------- rescale --
    const int et = threadIdx.x - 64;               // 0..127
    for (int i = et; i < nk * MT; i += 128) {      // scales of this CTA's K range
      const int kbi = i / MT, t = i % MT;
      xs_s[i] = t < M ? p.x_scale[static_cast<int64_t>(t) * p.xs_sm + static_cast<int64_t>(kb0 + kbi) * p.xs_sk]
                      : 0.0f;
    }
    for (int i = et; i < nk; i += 128) ws_s[i] = p.w_scale[static_cast<int64_t>(nt) * p.KB + kb0 + i];
    bar_sync(1, 128);
    const int q = warp & 3;                        // TMEM lane quarter of this warp
    const int row = q * 32 + lane;                 // weight row inside the tile
    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = 0.0f;
    bool done = true;
    for (int i = 0; i < nk; ++i) {
      const int buf = i % C::kBufs;
      const uint32_t bph = (i / C::kBufs) & 1;
      const bool got = wait_bounded(bar_tfull(buf), bph, abort_flag, status, kStEpilogue, tmo);
      if (!__all_sync(0xffffffffu, got)) {
        done = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * MT;
      uint32_t v[MT];
      if constexpr (MT == 16) {
        tmem_ld16(taddr, v);
      } else {
#pragma unroll
        for (int c = 0; c < MT / 32; ++c) tmem_ld32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + c * 32));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty(buf));  // the values are in registers: the buffer is free
      const float ws = ws_s[i];
      const float4* xs4 = reinterpret_cast<const float4*>(xs_s + i * MT);
#pragma unroll
      for (int t4 = 0; t4 < MT / 4; ++t4) {
        const float4 x = xs4[t4];
        acc[4 * t4 + 0] = fmaf(__uint_as_float(v[4 * t4 + 0]), x.x * ws, acc[4 * t4 + 0]);
        acc[4 * t4 + 1] = fmaf(__uint_as_float(v[4 * t4 + 1]), x.y * ws, acc[4 * t4 + 1]);
        acc[4 * t4 + 2] = fmaf(__uint_as_float(v[4 * t4 + 2]), x.z * ws, acc[4 * t4 + 2]);
        acc[4 * t4 + 3] = fmaf(__uint_as_float(v[4 * t4 + 3]), x.w * ws, acc[4 * t4 + 3]);
      }
    }
    if (done && *abort_flag == 0) {
      // token-major staging in the idle stage ring (every stage was consumed by
      // an MMA that completed before this warp's last wait)
      float* stg = reinterpret_cast<float*>(smem + C::kOffW);
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (t < M) stg[t * C::kPitch + row] = acc[t];
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
      const int first = produced > C::kStages ? produced - C::kStages : 0;
      volatile int no_abort = 0;
      for (int i = first; i < produced; ++i)
        wait_bounded(bar_full(i % C::kStages), (i / C::kStages) & 1, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      umma_commit(bar_drain);
      volatile int no_abort = 0;
      wait_bounded(bar_drain, 0, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  const bool ok = *abort_flag == 0;
  const int items = M * 32;                        // 4-column chunks of the M x 128 output block
  const float* stg = reinterpret_cast<const float*>(smem + C::kOffW);
  if (S == 1) {
    if (ok) {
      for (int it = threadIdx.x; it < items; it += C::kThreads) {
        const int t = it >> 5, c = (it & 31) * 4;
        const float4 v = *reinterpret_cast<const float4*>(stg + t * C::kPitch + c);
        store_out8(p, static_cast<int64_t>(t) * p.ldo + n0 + c, pack_bf16x4(v));
      }
      peer_store_fence(p);
    }
  } else {
    // split-K: every CTA of the cluster reaches both barriers, also after an
    // abort; each sums a disjoint range of the block's chunks over the slices in
    // order 0..S-1 (bitwise reproducible)
    cluster_sync_all();
    if (ok) {
      const int i0 = (s * items) / S, i1 = ((s + 1) * items) / S;
      const uint32_t sbase = base + C::kOffW;
      for (int it = i0 + static_cast<int>(threadIdx.x); it < i1; it += C::kThreads) {
        const int t = it >> 5, c = (it & 31) * 4;
        const uint32_t addr = sbase + static_cast<uint32_t>((t * C::kPitch + c) * 4);
        float4 sum = dsmem_ld4(dsmem_map(addr, 0));
        for (int r = 1; r < S; ++r) {
          const float4 v = dsmem_ld4(dsmem_map(addr, r));
          sum.x += v.x;
          sum.y += v.y;
          sum.z += v.z;
          sum.w += v.w;
        }
        store_out8(p, static_cast<int64_t>(t) * p.ldo + n0 + c, pack_bf16x4(sum));
      }
      peer_store_fence(p);
    }
    cluster_sync_all();
  }
  if (p.xchg) xchg_complete(p, status);
}

// ------------------------------------------------ small M (warp-level MMA) --
// For a few tokens the call is the weight stream and its fixed cost, and the
// tensor-memory pipeline's fixed cost (descriptor fetch, barrier set-up, TMEM
// allocation, cluster launch and barriers, the split-K combine) is most of
// it.  This kernel has none of that.  A CTA owns 16 weight rows and all M <= 16
// tokens; its 8 warps split the K blocks.  Each warp streams its K blocks'
// 16 x 128 weight bytes and 16 x 128 token bytes through a kStages-deep ring
// of its own in shared memory (cp.async, 512 contiguous bytes per warp
// instruction, kStages - 1 K blocks in flight) and feeds them to warp-level
// MMAs (m16n8k32, e4m3 x e4m3 -> f32), one or two per 32-wide K step (tokens
// 0-7, 8-15).  Each K block's f32 tile is scaled by
// w_scale[n/128, kb] * x_scale[t, kb] (a table computed once into shared
// memory, zero for tokens >= M) and accumulated; the warps' partials are
// summed in shared memory in warp order (deterministic) and stored as bf16.
//
// The ring holds each 128-byte row with its 16-byte chunks swizzled, logical
// chunk c of row r at c ^ (r & 7) -- the packed weight layout as it is, row-
// major weights and tokens rearranged on the way in -- so that the fragment
// reads below are free of bank conflicts.  Operand placement: thread
// (g = lane/4, q = lane%4) takes logical chunks 2q and 2q+1 of weight rows g
// and g+8; in K step s (0..3) word s of chunk 2q is the MMA's A column block
// 4q.. (a0 for row g, a1 for row g+8) and word s of chunk 2q+1 the block
// 16+4q.. (a2, a3); the token operand takes the same words of the token's
// chunks 2q and 2q+1 (b0, b1) for token g (and g+8 in the second MMA).  Any
// one-to-one map of the K block's 128 positions onto the MMA's 4 x 32 gives
// the same sum as long as both operands share it.
struct SmallCfg {
  static constexpr int kThreads = 256;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kRows = 16;                          // weight rows per CTA = tokens at most
  static constexpr int kStages = 3;                         // ring depth per warp
  static constexpr int kStageBytes = 2 * kRows * kBlk;      // weights, then tokens: 16 rows x 128 B each
  static constexpr int kRingBytes = kWarps * kStages * kStageBytes;
  static constexpr int kPitch = kRows + 1;                  // partials: [warp][row][token], padded rows
  static constexpr int kMaxKb = kSmallMaxKb;
  static constexpr int kSmemBytes = kRingBytes + kMaxKb * kRows * 4;   // + the scale table [KB][16]
  static_assert(kWarps * kRows * kPitch * 4 <= kRingBytes, "partials reuse the ring");
  static_assert(kSmemBytes <= 113 * 1024, "two CTAs per SM");
};

__global__ void __launch_bounds__(SmallCfg::kThreads, 2)
gemm_bs_small_kernel(const uint8_t* __restrict__ xq, int64_t ldx, const uint8_t* __restrict__ wq,
                     const __grid_constant__ Params p) {
  using C = SmallCfg;
  extern __shared__ __align__(128) uint8_t small_smem[];
  float* scale_tab = reinterpret_cast<float*>(small_smem + C::kRingBytes);   // [KB][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int n0 = blockIdx.x * C::kRows;
  const int KB = p.KB;
  const int kb_begin = (warp * KB) / C::kWarps;
  const int nk = ((warp + 1) * KB) / C::kWarps - kb_begin;
  const bool two = p.M > 8;                          // tokens 8-15 take a second MMA

  // Copy side: lane -> row lr + 4k (k = 0..3) and logical-or-stored chunk lc.
  const int lr = lane >> 3, lc = lane & 7;
  const uint8_t* wsrc;
  int64_t w_row_step, w_kb_step;
  int w_dst_c;                                       // chunk position in the ring; -1: swizzle on the way in
  if (p.w_packed) {
    // tile (n0/128, kb) is 128 rows x 128 B, chunks already at c ^ (row & 7);
    // n0 is a multiple of 16, so a tile row and its CTA row agree mod 8
    wsrc = wq + static_cast<int64_t>(n0 >> 7) * KB * (kBlk * kBlk) + static_cast<int64_t>((n0 & 127) + lr) * kBlk +
           lc * 16;
    w_row_step = 4 * kBlk;
    w_kb_step = kBlk * kBlk;
    w_dst_c = lc;
  } else {
    wsrc = wq + static_cast<int64_t>(n0 + lr) * p.K + lc * 16;
    w_row_step = 4 * static_cast<int64_t>(p.K);
    w_kb_step = kBlk;
    w_dst_c = -1;                                    // swizzle on the way in
  }
  wsrc += static_cast<int64_t>(kb_begin) * w_kb_step;
  const uint8_t* xsrc = xq + static_cast<int64_t>(kb_begin) * kBlk + lc * 16;
  const uint32_t ring = smem_addr(small_smem) + warp * (C::kStages * C::kStageBytes);
  const uint8_t* ring_ptr = small_smem + warp * (C::kStages * C::kStageBytes);

  grid_dependency_wait();

  auto issue = [&](int i) {  // the i-th K block of this warp into stage i % kStages
    if (i < nk) {
      const uint32_t wdst = ring + (i % C::kStages) * C::kStageBytes;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = lr + 4 * k;
        const int pos = w_dst_c >= 0 ? w_dst_c : (lc ^ (r & 7));
        cp_async16_cg(wdst + r * kBlk + pos * 16, wsrc + static_cast<int64_t>(i) * w_kb_step + k * w_row_step);
        const uint32_t xdst = wdst + C::kRows * kBlk;
        const bool tok = r < p.M;
        const uint8_t* xs = tok ? xsrc + static_cast<int64_t>(r) * ldx + static_cast<int64_t>(i) * kBlk : xsrc;
        cp_async16_cg_fill(xdst + r * kBlk + (lc ^ (r & 7)) * 16, xs, tok ? 16u : 0u);
      }
    }
    cp_async_commit();  // one group per K block, empty past the end, so the counts below hold
  };
#pragma unroll
  for (int i = 0; i < C::kStages - 1; ++i) issue(i);

  {
    const float* ws_row = p.w_scale + static_cast<int64_t>(n0 >> 7) * KB;
    for (int i = threadIdx.x; i < KB * C::kRows; i += C::kThreads) {
      const int kb = i / C::kRows, t = i - kb * C::kRows;
      scale_tab[i] = t < p.M ? ws_row[kb] * p.x_scale[t * p.xs_sm + static_cast<int64_t>(kb) * p.xs_sk] : 0.f;
    }
  }
  __syncthreads();  // the scale table is whole

  // fragment side: this thread's chunks 2q, 2q+1 of row g (and g+8, which
  // shares g & 7) sit at byte offsets o_lo, o_hi of a row
  const int o_lo = ((2 * q) ^ (g & 7)) * 16, o_hi = ((2 * q + 1) ^ (g & 7)) * 16;
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int i = 0; i < nk; ++i) {
    __syncwarp();                                    // every lane has read the stage refilled next
    issue(i + C::kStages - 1);
    cp_async_wait<C::kStages - 1>();                 // this lane's copies of K block i have landed ...
    __syncwarp();                                    // ... and every other lane's
    const uint8_t* w = ring_ptr + (i % C::kStages) * C::kStageBytes;
    const uint8_t* x = w + C::kRows * kBlk;         // the tokens' rows (zeros past M)
    const uint4 wa0 = *reinterpret_cast<const uint4*>(w + g * kBlk + o_lo);
    const uint4 wa1 = *reinterpret_cast<const uint4*>(w + g * kBlk + o_hi);
    const uint4 wb0 = *reinterpret_cast<const uint4*>(w + (g + 8) * kBlk + o_lo);
    const uint4 wb1 = *reinterpret_cast<const uint4*>(w + (g + 8) * kBlk + o_hi);
    const int kb = kb_begin + i;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (j == 1 && !two) break;
      const uint4 x0 = *reinterpret_cast<const uint4*>(x + (8 * j + g) * kBlk + o_lo);
      const uint4 x1 = *reinterpret_cast<const uint4*>(x + (8 * j + g) * kBlk + o_hi);
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      mma_e4m3_m16n8k32(d, wa0.x, wb0.x, wa1.x, wb1.x, x0.x, x1.x);
      mma_e4m3_m16n8k32(d, wa0.y, wb0.y, wa1.y, wb1.y, x0.y, x1.y);
      mma_e4m3_m16n8k32(d, wa0.z, wb0.z, wa1.z, wb1.z, x0.z, x1.z);
      mma_e4m3_m16n8k32(d, wa0.w, wb0.w, wa1.w, wb1.w, x0.w, x1.w);
      // d0, d1: row g, tokens 8j+2q, 8j+2q+1; d2, d3: row g+8, the same tokens
      const float2 sc = *reinterpret_cast<const float2*>(scale_tab + kb * C::kRows + 8 * j + 2 * q);
      acc[j][0] = fmaf(d[0], sc.x, acc[j][0]);
      acc[j][1] = fmaf(d[1], sc.y, acc[j][1]);
      acc[j][2] = fmaf(d[2], sc.x, acc[j][2]);
      acc[j][3] = fmaf(d[3], sc.y, acc[j][3]);
    }
  }
  cp_async_wait<0>();
  grid_launch_dependents();

  __syncthreads();  // every warp is done with the ring, which now holds the partials
  float* red = reinterpret_cast<float*>(small_smem);  // [warp][row * kPitch + token]
  float* mine = red + warp * (C::kRows * C::kPitch);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int t0 = 8 * j + 2 * q;
    mine[g * C::kPitch + t0] = acc[j][0];
    mine[g * C::kPitch + t0 + 1] = acc[j][1];
    mine[(g + 8) * C::kPitch + t0] = acc[j][2];
    mine[(g + 8) * C::kPitch + t0 + 1] = acc[j][3];
  }
  __syncthreads();
  // thread -> (token t, rows r, r+1): 8 threads cover a token's 16 rows
  const int t = threadIdx.x >> 3, r = (threadIdx.x & 7) * 2;
  if (t < p.M && t < C::kRows) {
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int w = 0; w < C::kWarps; ++w) {
      y0 += red[w * (C::kRows * C::kPitch) + r * C::kPitch + t];
      y1 += red[w * (C::kRows * C::kPitch) + (r + 1) * C::kPitch + t];
    }
    const __nv_bfloat162 b = __floats2bfloat162_rn(y0, y1);
    store_out4(p, static_cast<int64_t>(t) * p.ldo + n0 + r, *reinterpret_cast<const uint32_t*>(&b));
  }
  peer_store_fence(p);
  if (p.xchg) xchg_complete(p, &g_status);
}

// A stand-alone exchange step (one thread): orders a rank's next peer stores
// after everything its stream did before, on every rank.
__global__ void xchg_barrier_kernel(XchgState* x, Params pd, uint64_t timeout_ns) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    xchg_post(pd.peer_done, pd.n_peer, 0, 1);
    xchg_wait(x, pd.rank, pd.world, timeout_ns, &g_status);
  }
}

// ------------------------------------------------------------------ prepack --
// Tile (nb,kb) of WQ -> 16 KB block at ((nb*KB)+kb)*16384 holding the
// 128-byte-swizzled image: byte (r,c) of the tile at r*128 + ((c/16 ^ r%8)*16) + c%16.
__global__ void prepack_w_kernel(const uint8_t* __restrict__ w, int64_t ldw, int N, int K,
                                 uint8_t* __restrict__ out) {
  const int KB = K / kBlk;
  const int64_t total = static_cast<int64_t>(N) * (K / 16);  // 16-byte chunks
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = c / (K / 16);
    const int kc = static_cast<int>(c % (K / 16));     // 16-byte chunk along K
    const int kb = kc >> 3, ch = kc & 7;
    const int nb = static_cast<int>(n >> 7), r = static_cast<int>(n & 127);
    const uint4 v = *reinterpret_cast<const uint4*>(w + n * ldw + kc * 16);
    const int64_t dst = ((static_cast<int64_t>(nb) * KB + kb) * 128 + r) * 128 + ((ch ^ (r & 7)) << 4);
    *reinterpret_cast<uint4*>(out + dst) = v;
  }
}

// --------------------------------------------------------------- interleave --
__global__ void interleave_kernel(const __nv_bfloat16* __restrict__ g, int G, int M, int ns,
                                  __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t per_row = ns / 8;                                   // 16-byte chunks per shard row
  const int64_t total = static_cast<int64_t>(G) * M * per_row;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = c / (static_cast<int64_t>(M) * per_row);
    const int64_t rem = c % (static_cast<int64_t>(M) * per_row);
    const int64_t m = rem / per_row;
    const int64_t cc = rem % per_row;
    const uint4 v = *reinterpret_cast<const uint4*>(g + (r * M + m) * ns + cc * 8);
    *reinterpret_cast<uint4*>(out + m * ldo + r * ns + cc * 8) = v;
  }
}

// ===================================================================== host ==

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;

// weight tiles 64, 128, 256 x (single CTA, CTA pair) + swapped 16/32/64-token
// tiles + the persistent single-CTA kernel for weight tiles 64, 128, 256, 224
// + the warp-MMA small-M kernel for up to 16 tokens (16-row weight tiles)
constexpr int kVariants = 14;

static int variant(int tm, int bn) {
  if (bn == kSmallRows) return 13;
  if (tm < kTileM) return 6 + (tm == 16 ? 0 : tm == 32 ? 1 : 2);
  return (bn == 64 ? 0 : bn == 128 ? 1 : 2) + (tm == 256 ? 3 : 0);
}
static int persistent_variant(int bn) { return 9 + (bn == 64 ? 0 : bn == 128 ? 1 : bn == 256 ? 2 : 3); }

// Unsplit 128-token plans with more tiles than SMs run on the persistent
// kernel; FACK_PERSISTENT=0 in the environment keeps them on the one-tile
// kernel (the two give bitwise identical results).  224-wide weight tiles
// exist only in the persistent kernel and always run there.
static bool persistent_enabled() {
  static const bool on = [] {
    const char* e = getenv("FACK_PERSISTENT");
    return !(e && e[0] == '0');
  }();
  return on;
}

struct DeviceInfo {
  bool init = false;
  bool sm100 = false;
  int sms = 0;
  unsigned configured = 0;                       // bit per variant: attributes checked and set
  int clusters[kVariants][kMaxSplit + 1] = {};   // max co-resident clusters per (variant, split); 0 = unknown
};

static std::mutex g_mu;
static thread_local char g_last_error[256] = "";

// Records why a call failed (for fack_last_error) and returns `status`.
static int fail(int status, const char* what, cudaError_t err = cudaSuccess) {
  if (err != cudaSuccess)
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
  else
    snprintf(g_last_error, sizeof(g_last_error), "%s", what);
  return status;
}
int record_error(int status, const char* what) { return fail(status, what); }

static DeviceInfo g_dev[kMaxDevices];
static EncodeTiledFn g_encode = nullptr;

static int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= kMaxDevices) return FACK_ERR_CUDA;
  return FACK_OK;
}

static int device_info(DeviceInfo** out) {
  int dev;
  if (current_device(&dev) != FACK_OK) return FACK_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return FACK_ERR_CUDA;
    d.sm100 = (major == 10 && minor == 0);
    d.sms = sms;
    d.init = true;
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return FACK_ERR_CUDA;
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = &d;
  return d.sm100 ? FACK_OK : FACK_ERR_UNSUPPORTED_ARCH;
}

struct KernelEntry {
  const void* fn;
  int smem;
  int threads;
  bool split_regs;  // launched for the setmaxnreg split (exactly kLaunchRegs registers)
};

template <int BN, bool PAIR>
static KernelEntry entry() {
  return {reinterpret_cast<const void*>(gemm_bs_kernel<BN, PAIR>), Cfg<BN, PAIR>::kSmemBytes, kThreads, true};
}

template <int MT>
static KernelEntry swap_entry() {
  return {reinterpret_cast<const void*>(gemm_bs_swap_kernel<MT>), SwapCfg<MT>::kSmemBytes, SwapCfg<MT>::kThreads,
          false};
}

template <int BN>
static KernelEntry persistent_entry() {
  return {reinterpret_cast<const void*>(gemm_bs_persistent_kernel<BN>), PCfg<BN>::kSmemBytes, kThreads, true};
}

static KernelEntry small_entry() {
  return {reinterpret_cast<const void*>(gemm_bs_small_kernel), SmallCfg::kSmemBytes, SmallCfg::kThreads, false};
}

static const KernelEntry& kernel_by_variant(int v) {
  static const KernelEntry table[kVariants] = {
      entry<64, false>(),       entry<128, false>(),       entry<256, false>(),
      entry<64, true>(),        entry<128, true>(),        entry<256, true>(),
      swap_entry<16>(),         swap_entry<32>(),          swap_entry<64>(),
      persistent_entry<64>(),   persistent_entry<128>(),   persistent_entry<256>(),
      persistent_entry<224>(),  small_entry()};
  return table[v];
}

static const KernelEntry& kernel_for(int tm, int bn) { return kernel_by_variant(variant(tm, bn)); }

static int ensure_variant(DeviceInfo* d, int v) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!(d->configured & (1u << v))) {
    const KernelEntry& k = kernel_by_variant(v);
    // The setmaxnreg split assumes exactly kLaunchRegs registers per thread at
    // launch; with any other count setmaxnreg.inc could wait forever, so the
    // kernel is refused instead of launched.
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, k.fn);
    if (e != cudaSuccess) return fail(FACK_ERR_LAUNCH, "cudaFuncGetAttributes", e);
    if (k.split_regs && (fa.numRegs != kLaunchRegs || fa.maxThreadsPerBlock < kThreads))
      return fail(FACK_ERR_LAUNCH, "kernel register count differs from the setmaxnreg budget; refusing to launch");
    if (fa.maxThreadsPerBlock < k.threads) return fail(FACK_ERR_LAUNCH, "kernel cannot run its block size");
    e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
    if (e != cudaSuccess) return fail(FACK_ERR_LAUNCH, "cudaFuncSetAttribute(max dynamic shared memory)", e);
    d->configured |= 1u << v;
  }
  return FACK_OK;
}

static int ensure_configured(DeviceInfo* d, int tm, int bn) { return ensure_variant(d, variant(tm, bn)); }

// How many clusters of the (tm, bn) variant with `split` K slices the device
// holds at once.  A cluster is (tm/128, 1, split) CTAs and must fit inside
// one GPC, so on B200 fewer than 148/size clusters of a size fit.
static int co_resident(DeviceInfo* d, int tm, int bn, int split) {
  const int v = variant(tm, bn);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (d->clusters[v][split]) return d->clusters[v][split];
  }
  if (ensure_configured(d, tm, bn) != FACK_OK) return 0;
  const KernelEntry& k = kernel_for(tm, bn);
  const int cx = tm == 256 ? 2 : 1;  // pairs along cluster x
  int n = 0;
  if (split == 1 && cx == 1) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k.fn, k.threads, k.smem) != cudaSuccess) return 0;
    n = per_sm * d->sms;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cx, 1, split);
    cfg.blockDim = dim3(k.threads, 1, 1);
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

// Grid of a plan.  Single CTAs: x = weight tiles, y = 128-token tiles.  CTA
// pairs: x = 128-token tiles (an even count; a pair's second CTA may hold no
// valid token) so that the pair lies along the cluster's x dimension,
// y = weight tiles.  z = K slices.
static void plan_grid(int M, int N, int tm, int bn, int sp, int* gx, int* gy, int* gz) {
  if (bn == kSmallRows) {  // warp-MMA small-M kernel: x = 16-row weight tiles, K split inside the CTA
    *gx = N / kSmallRows;
    *gy = 1;
    *gz = 1;
    return;
  }
  if (tm < kTileM) {  // swapped small-M tiles: x = 128-row weight tiles
    *gx = N / kBlk;
    *gy = 1;
    *gz = sp;
    return;
  }
  if (tm == 256) {
    *gx = 2 * ((M + 255) / 256);
    *gy = N / bn;
  } else {
    *gx = N / bn;
    *gy = (M + kTileM - 1) / kTileM;
  }
  *gz = sp;
}

// Plan (token tile tm = 128 | 256 for a CTA pair, weight tile bn, split-K sp):
// the stand-in for aiter's tuned (M,N,K,cu_num) table.  Estimated launch time
// in SM cycles from per-SM rates measured on B200:
//  * a K block costs the slowest of: operand ingest (TMA fill into shared
//    memory, ~44 B/clk sustained per SM), the MMA (2*bn cycles for 128 rows),
//    and the MMA -> rescale -> TMEM-release round trip, which 512 TMEM
//    columns cannot hide at full MMA rate (~880 / 550 / 500 cycles for
//    bn = 256 / 128 / 64);
//  * per CTA ~4000 cycles of prologue, first-load latency and exit;
//  * output: bf16 tile stores at ~24 B/clk (the SM's store path), or for
//    split-K the exchange of (S-1)/S of the fp32 partial tile at ~18 B/clk
//    plus two cluster barriers;
// times the number of waves of co-resident clusters, bounded below by the HBM
// time of the operands.
static double plan_cost(DeviceInfo* d, int M, int N, int K, int tm, int bn, int sp) {
  const int KB = K / kBlk;
  if (bn == kSmallRows) {
    // warp-MMA small-M kernel: the weight stream at HBM speed, plus the
    // first loads' latency and exit; no pipeline to fill, no split-K combine
    (void)d;
    (void)sp;
    (void)KB;
    const double bytes = static_cast<double>(N) * K + static_cast<double>(M) * K;
    return bytes / 6.5e12 * 1.9e9 + 2500.0;
  }
  if (tm < kTileM) {
    // swapped small-M tiles: 128 weight rows x tm tokens; eight TMEM buffers
    // hide the rescale, so a K block costs the fill (weight tile + token
    // tile) or the narrow MMA (~226 cycles), whichever is slower
    const int tiles = N / kBlk;
    const int slots = co_resident(d, tm, kBlk, sp);                 // clusters of sp K slices
    if (slots <= 0) return 1e30;
    // one wave only: with more weight tiles than co-resident clusters (a
    // wide layer) the 128 x 256 tiles of the regular kernel measure faster
    if (tiles > slots) return 1e30;
    const int waves = 1;
    const int steps = (KB + sp - 1) / sp;
    const double t_kb = fmax((128.0 * 128.0 + tm * 128.0) / 44.0, 226.0);
    const double out = sp > 1 ? tm * 128.0 * 4.0 * (sp - 1) / sp / 18.0 + 2500.0 : M * 128.0 * 2.0 / 24.0;
    const double cyc = static_cast<double>(waves) * (steps * t_kb + 4000.0 + out);
    const double bytes = static_cast<double>(N) * K + static_cast<double>(M) * K;
    return fmax(cyc, bytes / 6.5e12 * 1.9e9);
  }
  const int tiles = (N / bn) * ((M + tm - 1) / tm) * (tm / kTileM);   // CTAs per K slice
  const int slots = co_resident(d, tm, bn, sp) * (tm / kTileM);       // CTAs per K slice resident at once
  if (slots <= 0) return 1e30;
  const int waves = (tiles + slots - 1) / slots;
  const int steps = (KB + sp - 1) / sp;
  const int rows = M < kTileM ? M : kTileM;                          // valid tokens of a full CTA tile
  const double wrows = tm == 256 ? bn / 2.0 : bn;
  const double ingest = (kTileM * 128.0 + wrows * 128.0) / 44.0;
  const double handshake = bn >= 224 ? 880.0 : bn >= 128 ? 550.0 : 500.0;
  const double t_kb = fmax(fmax(ingest, 2.0 * bn), handshake);
  const double out = sp > 1 ? rows * bn * 4.0 * (sp - 1) / sp / 18.0 + 2500.0 : rows * bn * 2.0 / 24.0;
  const double cyc = static_cast<double>(waves) * (steps * t_kb + 4000.0 + out);
  const double bytes = static_cast<double>(N) * K + static_cast<double>(M) * K;
  return fmax(cyc, bytes / 6.5e12 * 1.9e9);
}

// Tiles for an explicitly requested split (no device query, so the workspace
// size of an explicit split is a pure function of the shape): single-CTA
// token tiles unless pairs are requested, then the largest weight tile that
// still gives >= 120 CTAs, else the smallest.
static void tiles_for_split(int M, int N, int sp, int tm_req, int bn_req, int* tm, int* bn) {
  if (tm_req && tm_req < kTileM) {  // swapped small-M tiles span 128 weight rows, the warp-MMA ones 16
    *tm = tm_req;
    *bn = bn_req == kSmallRows ? kSmallRows : kBlk;
    return;
  }
  int t = tm_req ? tm_req : 128;
  int b = bn_req;
  if (!b) {
    b = 64;
    for (int c : {256, 128}) {
      int gx, gy, gz;
      if (N % c) continue;
      plan_grid(M, N, t, c, sp, &gx, &gy, &gz);
      if (gx * gy * gz >= 120) {
        b = c;
        break;
      }
    }
  }
  *tm = t;
  *bn = b;
}

static size_t workspace_bytes_for(int M, int N, int tm, int bn, int split);

// Best plan by plan_cost among those whose split-K workspace (when combined
// through global memory) is at most ws_cap bytes.
static int plan_auto(DeviceInfo* d, int M, int N, int K, int tm_req, int bn_req, int* tm_out, int* bn_out,
                     int* sp_out, size_t ws_cap = ~size_t(0)) {
  const int KB = K / kBlk;
  double best = 1e30;
  int bt = 0, bb = 0, bs = 0;
  // CTA pairs are chosen only on request for now: their cross-CTA handshakes
  // currently cost more per K block than the weight bytes they save.
  // swapped small-M tiles: the requested one, else the smallest token tile
  // that holds all M tokens
  const int tm_swap = tm_req && tm_req < kTileM ? tm_req : tm_req ? 0 : M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 0;
  // The warp-MMA small-M kernel, when no tile is requested (a requested
  // 16-token tile alone means the swapped kernel).  Paired A/B at K = 7168
  // on B200: faster than the swapped
  // 16 x 128 tiles at M <= 8 for every N (1.07-1.10x at N = 3072) and at
  // M <= 16 for N >= 8192 (1.10-1.12x), and than the 128 x 256 tiles by
  // 1.13-1.51x at N = 8192-16384 (even at 65536); the swapped kernel keeps
  // 9 <= M <= 16 at N <= 4096 (16 x 3072: 8.5 against 9.1 us).
  if (!tm_req && !bn_req && M <= 16 && KB <= kSmallMaxKb && (M <= 8 || N > 4096)) {
    *tm_out = 16;
    *bn_out = kSmallRows;
    *sp_out = 1;
    return FACK_OK;
  }
  if (tm_swap && M <= tm_swap && (bn_req == 0 || bn_req == kBlk)) {
    for (int sp = 1; sp <= KB && sp <= kMaxSplit; ++sp) {
      if ((KB + sp - 1) / sp > kSwapMaxKb) continue;
      if (sp > 1 && KB / sp < 2) break;
      const double c = plan_cost(d, M, N, K, tm_swap, kBlk, sp);
      if (c < best * 0.97) {
        best = c;
        bt = tm_swap;
        bb = kBlk;
        bs = sp;
      }
    }
  }
  for (int tm : {128, 256}) {
    if (tm_req ? tm != tm_req : tm != 128) continue;
    for (int bn : {256, 128, 64}) {
      if (N % bn || (bn_req && bn != bn_req)) continue;
      for (int sp = 1; sp <= KB && sp * (tm / kTileM) <= kMaxSplit; ++sp) {
        if (sp > 1 && KB / sp < 2) break;
        if (workspace_bytes_for(M, N, tm, bn, sp) > ws_cap) continue;
        const double c = plan_cost(d, M, N, K, tm, bn, sp);
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
  *tm_out = bt;
  *bn_out = bb;
  *sp_out = bs;
  return FACK_OK;
}

static size_t workspace_bytes_for(int M, int N, int tm, int bn, int split) {
  if (split <= 1 || tm < kTileM) return 0;  // small-M plans combine on chip only
  int gx, gy, gz;
  plan_grid(M, N, tm, bn, split, &gx, &gy, &gz);
  return static_cast<size_t>(gx) * gy * split * kTileM * bn * sizeof(float);
}

static int encode_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw,
                     CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_128B) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, promo,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FACK_OK : FACK_ERR_BAD_ALIGN;
}


// Tail split of a persistent launch of T tiles on G CTAs: the last rem = T % G
// tiles are cut into S K slices each (2 <= S <= 8, at least 2 K blocks per
// slice, rem * S <= G), so every CTA has at most one extra piece instead of a
// last round of rem whole tiles.  S = 0: no split (none needed or possible).
static void tail_schedule(int64_t T, int G, int KB, int* rem, int* S) {
  *rem = static_cast<int>(T % G);
  *S = 0;
  if (*rem == 0) return;
  int sp = G / *rem;
  if (sp > kMaxTailSplit) sp = kMaxTailSplit;
  if (sp > KB / 2) sp = KB / 2;
  if (sp >= 2) *S = sp;
}

static size_t tail_bytes(int rem, int S, int bn) {
  return static_cast<size_t>(rem) * S * kTileM * bn * sizeof(float);
}

static bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

template <int BN>
static const void* fixup_fn() {
  return reinterpret_cast<const void*>(gemm_bs_tail_fixup_kernel<BN>);
}

// `ws_bytes`: bytes at p.partials (0 without a workspace).  A persistent
// launch uses the workspace for its tail split when it holds the tail's
// partials, and then a fix-up launch follows in the same stream.
static int launch(DeviceInfo* d, int tm, int bn, const CUtensorMap& tw, const CUtensorMap& tx, const Params& p,
                  int M, cudaStream_t stream, size_t ws_bytes) {
  int gx, gy, gz;
  plan_grid(M, p.N, tm, bn, p.split, &gx, &gy, &gz);
  if (gy > 65535 || gz > 65535) return fail(FACK_ERR_BAD_SHAPE, "problem too large for one launch (grid y > 65535)");
  // more unsplit single-CTA tiles than SMs: one persistent CTA per SM
  const int64_t tiles = static_cast<int64_t>(gx) * gy;
  const bool persistent = tm == kTileM && p.split == 1 && (bn == 224 || (persistent_enabled() && tiles > d->sms));
  const int v = persistent ? persistent_variant(bn) : variant(tm, bn);
  const int st = ensure_variant(d, v);
  if (st != FACK_OK) return st;
  const KernelEntry& k = kernel_by_variant(v);
  Params q = p;
  q.tail_rem = 0;
  q.tail_split = 0;
  bool fixup = false;
  if (persistent) {
    gx = tiles < d->sms ? static_cast<int>(tiles) : d->sms;
    gy = 1;
    gz = 1;
    int rem = 0, S = 0;
    tail_schedule(tiles, d->sms, p.KB, &rem, &S);
    if (S && p.partials && aligned(p.partials, 16) && ws_bytes >= tail_bytes(rem, S, bn)) {
      q.tail_rem = rem;
      q.tail_split = S;
      q.xchg = nullptr;  // the fix-up launch, which stores the tail tiles, runs the exchange step
      fixup = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, gy, gz);
  cfg.blockDim = dim3(k.threads, 1, 1);
  cfg.dynamicSmemBytes = k.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  // programmatic dependent launch: this kernel's prologue may overlap the
  // previous kernel in the stream (see grid_dependency_wait in the kernel)
  attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
  ++cfg.numAttrs;
  if (p.split > 1 || tm == 256) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = tm == 256 ? 2 : 1;  // CTA pairs lie along cluster x
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = p.split;
    ++cfg.numAttrs;
  }
  void* args[] = {const_cast<CUtensorMap*>(&tw), const_cast<CUtensorMap*>(&tx), &q};
  cudaError_t e = cudaLaunchKernelExC(&cfg, k.fn, args);
  if (e != cudaSuccess) return fail(FACK_ERR_LAUNCH, "cudaLaunchKernelExC", e);
  if (!fixup) return FACK_OK;

  // the tail tiles: rem tiles x `chunks` row blocks, about one CTA per SM
  Params f = q;
  f.xchg = p.xchg;
  int chunks = d->sms / q.tail_rem;
  if (chunks > 16) chunks = 16;
  if (chunks < 1) chunks = 1;
  // A plain launch, not a programmatic dependent one: paired A/B on B200
  // (prefill, sustained load) measured the tail split 3.8 % faster than no
  // split this way, and 1.4-1.8 % slower with the fix-up launched early.
  cudaLaunchConfig_t fc = {};
  fc.gridDim = dim3(q.tail_rem * chunks, 1, 1);
  fc.blockDim = dim3(kFixupThreads, 1, 1);
  fc.stream = stream;
  fc.attrs = nullptr;
  fc.numAttrs = 0;
  const void* ffn = bn == 64 ? fixup_fn<64>() : bn == 128 ? fixup_fn<128>() : bn == 224 ? fixup_fn<224>() : fixup_fn<256>();
  void* fargs[] = {&f, &chunks};
  e = cudaLaunchKernelExC(&fc, ffn, fargs);
  if (e != cudaSuccess) return fail(FACK_ERR_LAUNCH, "cudaLaunchKernelExC (tail fix-up)", e);
  return FACK_OK;
}

// The warp-MMA small-M kernel: one CTA per 16 weight rows, plain
// pointers instead of tensor maps, no cluster.
static int launch_small(DeviceInfo* d, int tm, const uint8_t* xq, int64_t ldx, const uint8_t* wq, const Params& p,
                        cudaStream_t stream) {
  const int v = variant(tm, kSmallRows);
  const int st = ensure_variant(d, v);
  if (st != FACK_OK) return st;
  const KernelEntry& k = kernel_by_variant(v);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.N / kSmallRows, 1, 1);
  cfg.blockDim = dim3(k.threads, 1, 1);
  // the cp.async ring and the scale table of this launch's K blocks
  cfg.dynamicSmemBytes = SmallCfg::kRingBytes + static_cast<size_t>(p.KB) * kSmallRows * sizeof(float);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Params q = p;
  void* args[] = {const_cast<uint8_t**>(&xq), &ldx, const_cast<uint8_t**>(&wq), &q};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, k.fn, args);
  return e == cudaSuccess ? FACK_OK : fail(FACK_ERR_LAUNCH, "cudaLaunchKernelExC (small M)", e);
}

// ------------------------------------------------------ no-alloc scratch --
// Split-K scratch for fack_gemm_bs_noalloc: part of the library's own device
// image, so it exists on every GPU that loads the library, from load until the
// process exits, and using it never allocates.  16 MiB covers the decode
// shapes up to M = 512 at N = 3072 with the library's own split choice.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];
static void* g_noalloc_ptr[kMaxDevices];  // device address of the buffer, resolved once per device

// The array's name in host code is only a host-side handle: its device
// address must be asked for, on the device in question, before a kernel may
// use it.  The first call on each device does that (a runtime query, not an
// allocation) and caches the answer.
static int noalloc_scratch(void** out) {
  int dev;
  if (current_device(&dev) != FACK_OK) return FACK_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return FACK_ERR_CUDA;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return FACK_OK;
}

}  // namespace fack

using namespace fack;

extern "C" {

const char* fack_status_string(int status) {
  switch (status) {
    case FACK_OK: return "ok";
    case FACK_ERR_BAD_SHAPE: return "bad shape: need M >= 1 and N, K positive multiples of 128";
    case FACK_ERR_BAD_ALIGN: return "bad pointer: NULL or misaligned (xq, wq, out need 16 B; scales 4 B)";
    case FACK_ERR_BAD_STRIDE: return "bad stride: ldx >= K and ldx % 16 == 0, ldo >= N and ldo % 8 == 0, scale strides >= 1";
    case FACK_ERR_WS_TOO_SMALL: return "split-K workspace missing, misaligned or too small";
    case FACK_ERR_LAUNCH: return "kernel launch failed";
    case FACK_ERR_UNSUPPORTED_ARCH: return "current device is not sm_100 (B200)";
    case FACK_ERR_BAD_ARG: return "invalid argument";
    case FACK_ERR_DEVICE_TIMEOUT: return "a kernel gave up on a bounded wait (device status set)";
    case FACK_ERR_CUDA: return "CUDA runtime query failed";
    case FACK_ERR_SCRATCH_LIMIT:
      return "problem needs more split-K scratch than the no-allocation entry point's built-in 16 MiB; "
             "use fack_gemm_bs with a caller-owned workspace or request a smaller split_k";
    default: return "unknown status";
  }
}

int fack_version(void) { return 100; }

const char* fack_last_error(void) { return g_last_error; }

int fack_gemm_bs_plan(int M, int N, int K, int tile_m_request, int tile_n_request, int split_k_request,
                      int* tile_m, int* tile_n, int* split_k, size_t* workspace_bytes) {
  if (M < 1 || N < kBlk || K < kBlk || N % kBlk || K % kBlk || M > kMaxM) return FACK_ERR_BAD_SHAPE;
  if (!tile_m || !tile_n || !split_k) return FACK_ERR_BAD_ARG;
  const int KB = K / kBlk;
  if (split_k_request < 0 || split_k_request > kMaxSplit || split_k_request > KB) return FACK_ERR_BAD_ARG;
  if (tile_m_request != 0 && tile_m_request != 16 && tile_m_request != 32 && tile_m_request != 64 &&
      tile_m_request != 128 && tile_m_request != 256)
    return FACK_ERR_BAD_ARG;
  if (tile_n_request == kSmallRows) {
    // the warp-MMA small-M kernel: up to 16 tokens, K split inside the CTA
    if (tile_m_request != 0 && tile_m_request != 16) return FACK_ERR_BAD_ARG;
    const int tm = 16;
    if (M > tm || split_k_request > 1 || KB > kSmallMaxKb) return FACK_ERR_BAD_ARG;
    *tile_m = tm;
    *tile_n = kSmallRows;
    *split_k = 1;
    if (workspace_bytes) *workspace_bytes = 0;
    return FACK_OK;
  }
  if (tile_m_request && tile_m_request < kTileM) {  // swapped small-M tiles
    if (M > tile_m_request || (tile_n_request && tile_n_request != kBlk)) return FACK_ERR_BAD_ARG;
    if (split_k_request && (KB + split_k_request - 1) / split_k_request > kSwapMaxKb) return FACK_ERR_BAD_ARG;
  }
  if (tile_n_request != 0 && tile_n_request != 64 && tile_n_request != 128 && tile_n_request != 224 &&
      tile_n_request != 256)
    return FACK_ERR_BAD_ARG;
  if (tile_n_request && N % tile_n_request) return FACK_ERR_BAD_ARG;
  // 224-wide weight tiles: single 128-token CTAs, one K slice (the persistent kernel only)
  if (tile_n_request == 224 && ((tile_m_request && tile_m_request != kTileM) || split_k_request > 1))
    return FACK_ERR_BAD_ARG;
  if (tile_n_request == 224) {
    tile_m_request = kTileM;
    split_k_request = 1;
  }
  if (tile_m_request == 256 && split_k_request * 2 > kMaxSplit) return FACK_ERR_BAD_ARG;  // cluster of 2 x split
  int tm = tile_m_request, bn = tile_n_request, sp = split_k_request;
  if (sp) {
    tiles_for_split(M, N, sp, tm, bn, &tm, &bn);
  } else {
    DeviceInfo* d = nullptr;
    const int st = device_info(&d);
    if (st != FACK_OK) return st;
    // an exact-shape row of the tuned table fixes a fully automatic plan
    if (tm || bn || !tuned_lookup(d->sms, M, N, K, &tm, &bn, &sp)) {
      const int st2 = plan_auto(d, M, N, K, tm, bn, &tm, &bn, &sp);
      if (st2 != FACK_OK) return st2;
    }
  }
  *tile_m = tm;
  *tile_n = bn;
  *split_k = sp;
  if (workspace_bytes) *workspace_bytes = workspace_bytes_for(M, N, tm, bn, sp);
  return FACK_OK;
}

int fack_gemm_bs_plan_estimate(int M, int N, int K, int tile_m, int tile_n, int split_k, double* cycles) {
  if (!cycles) return FACK_ERR_BAD_ARG;
  const int v = tuned_validate(M, N, K, tile_m, tile_n, split_k);  // the rules of an explicit plan
  if (v != FACK_OK) return v;
  DeviceInfo* d = nullptr;
  const int st = device_info(&d);
  if (st != FACK_OK) return st;
  *cycles = plan_cost(d, M, N, K, tile_m, tile_n, split_k);
  return FACK_OK;
}

int fack_gemm_bs_tail_workspace_size(int M, int N, int K, int tile_m_request, int tile_n_request,
                                     int split_k_request, size_t* bytes) {
  if (!bytes) return FACK_ERR_BAD_ARG;
  int tm = 0, bn = 0, sp = 0;
  size_t need = 0;
  int st = fack_gemm_bs_plan(M, N, K, tile_m_request, tile_n_request, split_k_request, &tm, &bn, &sp, &need);
  if (st != FACK_OK) return st;
  *bytes = 0;
  if (tm != kTileM || sp != 1 || !persistent_enabled()) return FACK_OK;
  DeviceInfo* d = nullptr;
  st = device_info(&d);
  if (st != FACK_OK) return st;
  int gx, gy, gz;
  plan_grid(M, N, tm, bn, sp, &gx, &gy, &gz);
  const int64_t tiles = static_cast<int64_t>(gx) * gy;
  if (tiles <= d->sms) return FACK_OK;
  int rem = 0, S = 0;
  tail_schedule(tiles, d->sms, K / kBlk, &rem, &S);
  if (S) *bytes = tail_bytes(rem, S, bn);
  return FACK_OK;
}

int fack_gemm_bs_select(int M, int N, int K, int split_k_request, int* tile_n, int* split_k) {
  int tm = 0;
  return fack_gemm_bs_plan(M, N, K, 0, 0, split_k_request, &tm, tile_n, split_k, nullptr);
}

int fack_gemm_bs_workspace_size(int M, int N, int K, int split_k, size_t* bytes) {
  if (!bytes) return FACK_ERR_BAD_ARG;
  int tm = 0, bn = 0, sp = 0;
  return fack_gemm_bs_plan(M, N, K, 0, 0, split_k, &tm, &bn, &sp, bytes);
}

int fack_gemm_bs_prepack_w(const void* wq, int64_t ldw, const float* w_scale, int N, int K, void* wq_packed,
                           float* ws_packed, void* stream) {
  if (N < kBlk || K < kBlk || N % kBlk || K % kBlk) return FACK_ERR_BAD_SHAPE;
  if (!wq || !wq_packed || !aligned(wq, 16) || !aligned(wq_packed, 16)) return FACK_ERR_BAD_ALIGN;
  if (ldw < K || ldw % 16) return FACK_ERR_BAD_STRIDE;
  if (ws_packed && (!w_scale || !aligned(w_scale, 4) || !aligned(ws_packed, 4))) return FACK_ERR_BAD_ALIGN;
  DeviceInfo* d = nullptr;
  const int st = device_info(&d);
  if (st != FACK_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t chunks = static_cast<int64_t>(N) * (K / 16);
  const int threads = 256;
  int64_t blocks = (chunks + threads - 1) / threads;
  if (blocks > 8 * d->sms * 8) blocks = 8 * d->sms * 8;
  prepack_w_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(static_cast<const uint8_t*>(wq), ldw, N, K,
                                                                     static_cast<uint8_t*>(wq_packed));
  if (cudaGetLastError() != cudaSuccess) return FACK_ERR_LAUNCH;
  if (ws_packed) {
    const size_t bytes = static_cast<size_t>(N / kBlk) * (K / kBlk) * sizeof(float);
    if (cudaMemcpyAsync(ws_packed, w_scale, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return FACK_ERR_LAUNCH;
  }
  return FACK_OK;
}

}  // extern "C"

// fack_gemm_bs_ex with the result also stored to n_peers peer copies of the
// output block (same ldo); n_peers = 0 is fack_gemm_bs_ex.
// With `xchg` (the fused all-gather: world - 1 peers, this rank's exchange
// state and each peer's mapped state, in rank order without `rank`) the
// launch also runs the completion step of xchg_complete.
static int gemm_bs_impl(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                        int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo,
                        void* const* peer_outs, int n_peers, int M, int N, int K, int tile_m, int tile_n,
                        int split_k, void* workspace, size_t workspace_bytes, void* stream, void* xchg = nullptr,
                        void* const* peer_xchg = nullptr, int rank = 0, int world = 1) {
  if (M < 1 || N < kBlk || K < kBlk || N % kBlk || K % kBlk) return FACK_ERR_BAD_SHAPE;
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peer_outs)) return FACK_ERR_BAD_ARG;
  for (int i = 0; i < n_peers; ++i)
    if (!peer_outs[i] || !aligned(peer_outs[i], 16)) return FACK_ERR_BAD_ALIGN;
  if (M > kMaxM) return FACK_ERR_BAD_SHAPE;
  if (wq_packed != FACK_W_ROW_MAJOR && wq_packed != FACK_W_PACKED) return FACK_ERR_BAD_ARG;
  if (!xq || !wq || !out || !x_scale || !w_scale) return FACK_ERR_BAD_ALIGN;
  if (!aligned(xq, 16) || !aligned(wq, 16) || !aligned(out, 16) || !aligned(x_scale, 4) || !aligned(w_scale, 4))
    return FACK_ERR_BAD_ALIGN;
  if (ldx < K || ldx % 16 || ldo < N || ldo % 8 || xs_stride_m < 1 || xs_stride_kb < 1) return FACK_ERR_BAD_STRIDE;
  const int KB = K / kBlk;
  if (split_k < 0 || split_k > kMaxSplit || split_k > KB) return FACK_ERR_BAD_ARG;

  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != FACK_OK) return st;
  int tm = 0, bn = 0, sp = 0;
  size_t need = 0;
  st = fack_gemm_bs_plan(M, N, K, tile_m, tile_n, split_k, &tm, &bn, &sp, &need);
  if (st != FACK_OK) return st;
  const int wrows = tm == 256 ? bn / 2 : bn;  // weight rows one CTA loads
  // A NULL workspace selects the distributed-shared-memory split-K reduction.
  if (need && workspace && (workspace_bytes < need || !aligned(workspace, 16))) return FACK_ERR_WS_TOO_SMALL;
  if (!workspace) workspace_bytes = 0;

  Params p;
  p.x_scale = x_scale;
  p.xs_sm = xs_stride_m;
  p.xs_sk = xs_stride_kb;
  p.w_scale = w_scale;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.n_peer = n_peers;
  for (int i = 0; i < kMaxPeers; ++i)
    p.peer_out[i] = i < n_peers ? static_cast<__nv_bfloat16*>(peer_outs[i]) : nullptr;
  p.partials = static_cast<float*>(workspace);
  p.M = M;
  p.N = N;
  p.K = K;
  p.KB = KB;
  p.split = sp;
  p.w_packed = wq_packed;
  p.timeout_ns = 2000000000ull;  // 2 s: far above any legitimate wait, short enough to report a lost arrival
  p.xchg = static_cast<XchgState*>(xchg);
  p.rank = rank;
  p.world = world;
  for (int i = 0; i < kMaxPeers; ++i) p.peer_done[i] = nullptr;
  if (xchg) {
    for (int i = 0; i < n_peers; ++i)
      p.peer_done[i] = reinterpret_cast<unsigned long long*>(static_cast<char*>(peer_xchg[i]) +
                                                             offsetof(XchgState, done)) + rank;
  }
  // a peer may legitimately start its step later than this rank (host-side
  // work between steps); 10 s bounds the wait for one that never comes
  p.xchg_timeout_ns = 10000000000ull;

  p.tail_rem = 0;
  p.tail_split = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bn == kSmallRows) return launch_small(d, tm, static_cast<const uint8_t*>(xq), ldx,
                                            static_cast<const uint8_t*>(wq), p, s);

  CUtensorMap tw, tx;
  if (wq_packed == FACK_W_PACKED)
    st = encode_2d(&tw, wq, kBlk, static_cast<uint64_t>(N) * KB, kBlk, kBlk,
                   wrows == 224 ? 32 : wrows < kBlk ? wrows : kBlk,   // 224-row tiles: seven 32-row boxes
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);  // packed tiles are contiguous
  else
    st = encode_2d(&tw, wq, K, N, K, kBlk, wrows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != FACK_OK) return st;
  st = encode_2d(&tx, xq, K, M, ldx, kBlk, tm < kTileM ? tm : kTileM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != FACK_OK) return st;

  return launch(d, tm, bn, tw, tx, p, M, s, workspace ? workspace_bytes : 0);
}

// Rules shared by the entry points of the fused all-gather.
static int check_exchange(void* xchg, void* const* peer_xchg, int rank, int world) {
  if (world < 2 || world > kMaxRanks || rank < 0 || rank >= world) return FACK_ERR_BAD_ARG;
  if (!peer_xchg) return FACK_ERR_BAD_ARG;
  if (!xchg || !aligned(xchg, 16)) return FACK_ERR_BAD_ALIGN;
  for (int i = 0; i < world - 1; ++i)
    if (!peer_xchg[i] || !aligned(peer_xchg[i], 16)) return FACK_ERR_BAD_ALIGN;
  return FACK_OK;
}

extern "C" {

int fack_gemm_bs_ex(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                    int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo, int M,
                    int N, int K, int tile_m, int tile_n, int split_k, void* workspace, size_t workspace_bytes,
                    void* stream) {
  return gemm_bs_impl(xq, ldx, wq, wq_packed, x_scale, xs_stride_m, xs_stride_kb, w_scale, out, ldo, nullptr, 0, M,
                      N, K, tile_m, tile_n, split_k, workspace, workspace_bytes, stream);
}

int fack_gemm_bs_bcast(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                       int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo,
                       void* const* peer_outs, int n_peers, int M, int N, int K, int tile_m, int tile_n, int split_k,
                       void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_bs_impl(xq, ldx, wq, wq_packed, x_scale, xs_stride_m, xs_stride_kb, w_scale, out, ldo, peer_outs,
                      n_peers, M, N, K, tile_m, tile_n, split_k, workspace, workspace_bytes, stream);
}

int fack_gemm_bs_allgather(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                           int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo,
                           void* const* peer_outs, void* xchg, void* const* peer_xchg, int rank, int world, int M,
                           int N, int K, int tile_m, int tile_n, int split_k, void* workspace,
                           size_t workspace_bytes, void* stream) {
  const int st = check_exchange(xchg, peer_xchg, rank, world);
  if (st != FACK_OK) return st;
  if (!peer_outs) return FACK_ERR_BAD_ARG;
  return gemm_bs_impl(xq, ldx, wq, wq_packed, x_scale, xs_stride_m, xs_stride_kb, w_scale, out, ldo, peer_outs,
                      world - 1, M, N, K, tile_m, tile_n, split_k, workspace, workspace_bytes, stream, xchg,
                      peer_xchg, rank, world);
}

int fack_xchg_barrier(void* xchg, void* const* peer_xchg, int rank, int world, void* stream) {
  const int st0 = check_exchange(xchg, peer_xchg, rank, world);
  if (st0 != FACK_OK) return st0;
  DeviceInfo* d = nullptr;
  const int st = device_info(&d);
  if (st != FACK_OK) return st;
  Params pd;
  memset(&pd, 0, sizeof(pd));
  pd.n_peer = world - 1;
  pd.rank = rank;
  pd.world = world;
  for (int i = 0; i < world - 1; ++i)
    pd.peer_done[i] = reinterpret_cast<unsigned long long*>(static_cast<char*>(peer_xchg[i]) +
                                                            offsetof(XchgState, done)) + rank;
  xchg_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<XchgState*>(xchg), pd,
                                                                        10000000000ull);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FACK_OK : fail(FACK_ERR_LAUNCH, "xchg_barrier_kernel", e);
}

// ------------------------------------------------------------ CUDA IPC --
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int fack_ipc_get_handle(const void* ptr, void* handle, size_t handle_bytes, size_t* offset) {
  if (!ptr || !handle || !offset || handle_bytes < sizeof(cudaIpcMemHandle_t)) return FACK_ERR_BAD_ARG;
  // looked up once; a function-local static is initialised thread-safely
  static const AddressRangeFn range = []() -> AddressRangeFn {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<AddressRangeFn>(fn);
  }();
  if (!range) return fail(FACK_ERR_CUDA, "cuMemGetAddressRange entry point");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(FACK_ERR_BAD_ARG, "pointer is not device memory");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(FACK_ERR_CUDA, "cudaIpcGetMemHandle", e);
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return FACK_OK;
}

int fack_ipc_open_handle(const void* handle, void** base) {
  if (!handle || !base) return FACK_ERR_BAD_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(FACK_ERR_CUDA, "cudaIpcOpenMemHandle", e);
  return FACK_OK;
}

int fack_ipc_close_handle(void* base) {
  if (!base) return FACK_ERR_BAD_ARG;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return fail(FACK_ERR_CUDA, "cudaIpcCloseMemHandle", e);
  return FACK_OK;
}

int fack_gemm_bs(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                 int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo, int M,
                 int N, int K, int split_k, void* workspace, size_t workspace_bytes, void* stream) {
  return fack_gemm_bs_ex(xq, ldx, wq, wq_packed, x_scale, xs_stride_m, xs_stride_kb, w_scale, out, ldo, M, N, K, 0,
                         0, split_k, workspace, workspace_bytes, stream);
}

int fack_gemm_bs_noalloc(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                         int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo,
                         int M, int N, int K, int split_k, void* stream) {
  int tm = 0, bn = 0, sp = 0;
  size_t need = 0;
  int st = fack_gemm_bs_plan(M, N, K, 0, 0, split_k, &tm, &bn, &sp, &need);
  if (st != FACK_OK) return st;
  if (need > kNoAllocScratchBytes && split_k == 0) {
    // the library's own choice: take the best plan whose partials fit the buffer
    DeviceInfo* d = nullptr;
    st = device_info(&d);
    if (st != FACK_OK) return st;
    st = plan_auto(d, M, N, K, 0, 0, &tm, &bn, &sp, kNoAllocScratchBytes);
    if (st != FACK_OK) return FACK_ERR_SCRATCH_LIMIT;
    need = workspace_bytes_for(M, N, tm, bn, sp);
  }
  if (need > kNoAllocScratchBytes) return FACK_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need) {
    st = noalloc_scratch(&scratch);
    if (st != FACK_OK) return st;
  }
  // The same kernel and plan as fack_gemm_bs; only the workspace differs.
  return fack_gemm_bs_ex(xq, ldx, wq, wq_packed, x_scale, xs_stride_m, xs_stride_kb, w_scale, out, ldo, M, N, K, tm,
                         bn, sp, scratch, need ? kNoAllocScratchBytes : 0, stream);
}

int fack_gather_interleave(const void* gathered, int g, int M, int n_shard, void* out, int64_t ldo, void* stream) {
  if (g < 1 || M < 1 || n_shard < 8 || n_shard % 8) return FACK_ERR_BAD_SHAPE;
  if (!gathered || !out || !aligned(gathered, 16) || !aligned(out, 16)) return FACK_ERR_BAD_ALIGN;
  if (ldo < static_cast<int64_t>(g) * n_shard || ldo % 8) return FACK_ERR_BAD_STRIDE;
  DeviceInfo* d = nullptr;
  const int st = device_info(&d);
  if (st != FACK_OK) return st;
  const int64_t chunks = static_cast<int64_t>(g) * M * (n_shard / 8);
  const int threads = 256;
  int64_t blocks = (chunks + threads - 1) / threads;
  if (blocks > 8 * d->sms * 8) blocks = 8 * d->sms * 8;
  interleave_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gathered), g, M, n_shard, static_cast<__nv_bfloat16*>(out), ldo);
  return cudaGetLastError() == cudaSuccess ? FACK_OK : FACK_ERR_LAUNCH;
}

}  // extern "C"

namespace fack {
// Device address of the status word on the current device, for the other
// kernels of the library that report bounded-wait timeouts through it.
unsigned int* device_status_word() {
  void* p = nullptr;
  return cudaGetSymbolAddress(&p, g_status) == cudaSuccess ? static_cast<unsigned int*>(p) : nullptr;
}

int sm100_device(int* sms) {
  DeviceInfo* d = nullptr;
  const int st = device_info(&d);
  if (st != FACK_OK) return st;
  *sms = d->sms;
  return FACK_OK;
}

int encode_bytes_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  return encode_2d(map, ptr, inner, outer, row_bytes, box_inner, box_outer,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}
}  // namespace fack

extern "C" {

int fack_device_status(void* stream, unsigned int* flags, int reset) {
  if (!flags) return FACK_ERR_BAD_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_status, sizeof(v), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return FACK_ERR_CUDA;
  if (reset) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return FACK_ERR_CUDA;
  }
  *flags = v;
  return v ? FACK_ERR_DEVICE_TIMEOUT : FACK_OK;
}

}  // extern "C"
