// gemm_bs_sm100.cu -- FP8 (e4m3) block-scaled GEMM for B200 (sm_100a).
//
//   Y[m,n] (bf16) = sum_kb (XQ[m,kb-block] . WQ[n,kb-block]) * x_scale[m,kb] * w_scale[n/128,kb]
//
// The arithmetic restated from client/aiter/hsa/gfx942/driver.py:18-20 (the
// reference's fp32 oracle for aiter's gemm_a8w8_blockscale_bpreshuffle_asm).
//
// Design (B200-first, not a translation of the gfx942 kernels):
//  * swap-AB: the 128 weight rows of a tile are the UMMA M side (TMEM lanes),
//    the tokens are the UMMA N side (TMEM columns, 32..256).  A 128-row weight
//    tile lies inside one 128x128 scale block, so w_scale is one scalar per
//    (tile, kb) and x_scale is one value per TMEM column.
//  * per 128-wide K block (kb): TMA brings a 128x128 B weight tile and a
//    BNx128 B token tile into a multi-stage mbarrier ring (128-byte swizzle);
//    one thread issues 4 tcgen05.mma (K=32 each) into one of two TMEM
//    buffers; 8 epilogue warps read the finished buffer with tcgen05.ld and
//    fold it into fp32 register accumulators with acc += partial *
//    (x_scale * w_scale) -- the per-block rescale cannot go into the MMA
//    because the scales are arbitrary fp32 values, not UE8M0 powers of two.
//    The double-buffered TMEM lets the MMA of kb+1 overlap the rescale of kb.
//  * split-K for small M: the K slices of one output tile form a thread-block
//    cluster along grid z.  Each CTA writes its fp32 partial tile to the
//    workspace, the cluster barrier publishes them, and each CTA then sums a
//    disjoint set of rows over all slices in slice order 0..S-1, so results
//    are bitwise reproducible and no CTA ever spins on another.
//  * every mbarrier wait is bounded by a %globaltimer deadline; on expiry the
//    CTA raises an abort flag, records a code in the device status word,
//    drains its in-flight TMA copies and MMAs, frees TMEM and exits.
//  * no TMA multicast anywhere: the same kernel serves the N-sharded
//    multi-GPU path.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/fack_gemm.h"
#include "sm100_ptx.cuh"

namespace fack {

constexpr int kBlk = 128;          // quantisation block along K and N
constexpr int kTileW = 128;        // weight rows per CTA (UMMA M)
constexpr int kThreads = 384;      // 12 warps
constexpr int kEpiWarp0 = 4;       // warps 4..11 rescale and store
constexpr int kEpiWarps = 8;
constexpr int kScaleRing = 4;      // depth of the combined-scale ring
constexpr int kMaxSplit = 8;       // portable cluster size
constexpr int kSmemBudget = 196608;

// Device status word: set by kernels whose bounded waits expired.
__device__ unsigned int g_status;

enum : unsigned int {
  kStProducer = 1u,
  kStMma = 2u,
  kStScale = 4u,
  kStEpilogue = 8u,
  kStDrain = 16u
};

template <int BN>
struct Cfg {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "token tile must be 32..256, multiple of 32");
  static constexpr int kABytes = kTileW * kBlk;            // 16 KB weight tile
  static constexpr int kBBytes = BN * kBlk;                 // token tile
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr int kTmemBuf = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int kTmemCols = 2 * kTmemBuf;            // power of two, >= 64
  static constexpr int kCpw = BN / 2;                       // columns per epilogue warp
  // shared-memory carve-up (offsets from a 1024-byte aligned base)
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kStages * kABytes;
  static constexpr int kOffScale = kOffB + kStages * kBBytes;
  static constexpr int kOffBar = kOffScale + kScaleRing * BN * 4;
  static constexpr int kNumBars = 2 * kStages + 4 + 2 * kScaleRing + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;   // + alignment slack
  static_assert(kStages >= 2, "pipeline needs two stages");
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
  static_assert(kStages * kABytes >= BN * kTileW * 2, "output staging must fit in the A ring");
};

struct Params {
  const float* x_scale;
  int64_t xs_sm, xs_sk;
  const float* w_scale;        // [N/128][K/128]
  __nv_bfloat16* out;
  int64_t ldo;
  float* partials;             // [tiles][S][BN][128] fp32, S > 1 only
  int M, N, K, KB;
  int split;
  int w_packed;
  uint64_t timeout_ns;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bs_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
               const __grid_constant__ Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int nt = blockIdx.x;                 // weight tile (128 output columns)
  const int mt = blockIdx.y;                 // token tile
  const int s = blockIdx.z;                  // K slice
  const int S = p.split;
  const int m0 = mt * BN;
  const int n0 = nt * kTileW;
  const int kb0 = (s * p.KB) / S;
  const int kb1 = ((s + 1) * p.KB) / S;
  const int nk = kb1 - kb0;

  float* csc = reinterpret_cast<float*>(smem + C::kOffScale);
  const uint32_t bar0 = base + C::kOffBar;
  auto bar_full = [&](int i) { return bar0 + 8u * i; };
  auto bar_empty = [&](int i) { return bar0 + 8u * (C::kStages + i); };
  auto bar_tfull = [&](int i) { return bar0 + 8u * (2 * C::kStages + i); };
  auto bar_tempty = [&](int i) { return bar0 + 8u * (2 * C::kStages + 2 + i); };
  auto bar_sfull = [&](int i) { return bar0 + 8u * (2 * C::kStages + 4 + i); };
  auto bar_sempty = [&](int i) { return bar0 + 8u * (2 * C::kStages + 4 + kScaleRing + i); };
  const uint32_t bar_drain = bar0 + 8u * (2 * C::kStages + 4 + 2 * kScaleRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(bar_full(i), 1);
      mbar_init(bar_empty(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_tfull(i), 1);
      mbar_init(bar_tempty(i), kEpiWarps);
    }
    for (int i = 0; i < kScaleRing; ++i) {
      mbar_init(bar_sfull(i), 32);
      mbar_init(bar_sempty(i), kEpiWarps);
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
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t tmo = p.timeout_ns;
  unsigned int* status = &g_status;

  int produced = 0;  // TMA stages issued (producer lane only)

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();   // weights stream once
      const uint64_t pol_x = policy_evict_last();    // tokens are re-read by every weight tile
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        if (!wait_bounded(bar_empty(st), ph ^ 1u, abort_flag, status, kStProducer, tmo)) break;
        const int kb = kb0 + i;
        mbar_arrive_expect_tx(bar_full(st), C::kStageBytes);
        const uint32_t sa = base + C::kOffA + st * C::kABytes;
        const uint32_t sb = base + C::kOffB + st * C::kBBytes;
        if (p.w_packed)
          tma_load_2d(sa, &tmap_w, bar_full(st), 0, (nt * p.KB + kb) * kBlk, pol_w);
        else
          tma_load_2d(sa, &tmap_w, bar_full(st), kb * kBlk, n0, pol_w);
        tma_load_2d(sb, &tmap_x, bar_full(st), kb * kBlk, m0, pol_x);
        produced = i + 1;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(kTileW, BN);
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        const uint32_t ph = (i / C::kStages) & 1;
        const int buf = i & 1;
        const uint32_t bph = (i >> 1) & 1;
        if (!wait_bounded(bar_tempty(buf), bph ^ 1u, abort_flag, status, kStMma, tmo)) break;
        if (!wait_bounded(bar_full(st), ph, abort_flag, status, kStMma, tmo)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + buf * C::kTmemBuf;
        const uint64_t da = sw128_kmajor_desc(base + C::kOffA + st * C::kABytes);
        const uint64_t db = sw128_kmajor_desc(base + C::kOffB + st * C::kBBytes);
#pragma unroll
        for (int k = 0; k < kBlk / 32; ++k)  // K = 32 e4m3 elements = 32 bytes = 2 descriptor units
          umma_f8(d, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
        umma_commit(bar_empty(st));
        umma_commit(bar_tfull(buf));
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------ combined-scale ring --
    const float* wsc = p.w_scale + static_cast<int64_t>(nt) * p.KB;
    for (int i = 0; i < nk; ++i) {
      const int r = i % kScaleRing;
      const uint32_t ph = (i / kScaleRing) & 1;
      if (!wait_bounded(bar_sempty(r), ph ^ 1u, abort_flag, status, kStScale, tmo)) break;
      const int kb = kb0 + i;
      const float sw = __ldg(wsc + kb);
      float* dst = csc + r * BN;
      for (int j = lane; j < BN; j += 32) {
        const int m = m0 + j;
        dst[j] = (m < p.M) ? __ldg(p.x_scale + m * p.xs_sm + kb * p.xs_sk) * sw : 0.0f;
      }
      mbar_arrive(bar_sfull(r));
    }
  }

  // ------------------------------------------------------------ epilogue --
  float acc[C::kCpw];
  const bool is_epi = warp >= kEpiWarp0;
  const int q = warp & 3;                       // TMEM lane quarter this warp may access
  const int h = (warp - kEpiWarp0) >> 2;        // column half
  const int col0 = h * C::kCpw;
  if (is_epi) {
#pragma unroll
    for (int j = 0; j < C::kCpw; ++j) acc[j] = 0.0f;
    for (int i = 0; i < nk; ++i) {
      const int buf = i & 1;
      const uint32_t bph = (i >> 1) & 1;
      const int r = i % kScaleRing;
      const uint32_t sph = (i / kScaleRing) & 1;
      // tcgen05.ld is .sync.aligned: the whole warp must agree before using it.
      bool got = wait_bounded(bar_tfull(buf), bph, abort_flag, status, kStEpilogue, tmo);
      got = got && wait_bounded(bar_sfull(r), sph, abort_flag, status, kStEpilogue, tmo);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * C::kTmemBuf + col0;
      const float4* sc = reinterpret_cast<const float4*>(csc + r * BN + col0);
#pragma unroll
      for (int c = 0; c + 32 <= C::kCpw; c += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + c, v);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float4 f = sc[(c >> 2) + t];
          acc[c + 4 * t + 0] = fmaf(__uint_as_float(v[4 * t + 0]), f.x, acc[c + 4 * t + 0]);
          acc[c + 4 * t + 1] = fmaf(__uint_as_float(v[4 * t + 1]), f.y, acc[c + 4 * t + 1]);
          acc[c + 4 * t + 2] = fmaf(__uint_as_float(v[4 * t + 2]), f.z, acc[c + 4 * t + 2]);
          acc[c + 4 * t + 3] = fmaf(__uint_as_float(v[4 * t + 3]), f.w, acc[c + 4 * t + 3]);
        }
      }
      if constexpr (C::kCpw % 32 == 16) {
        constexpr int c = C::kCpw - 16;
        uint32_t v[16];
        tmem_ld16(taddr + c, v);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float4 f = sc[(c >> 2) + t];
          acc[c + 4 * t + 0] = fmaf(__uint_as_float(v[4 * t + 0]), f.x, acc[c + 4 * t + 0]);
          acc[c + 4 * t + 1] = fmaf(__uint_as_float(v[4 * t + 1]), f.y, acc[c + 4 * t + 1]);
          acc[c + 4 * t + 2] = fmaf(__uint_as_float(v[4 * t + 2]), f.z, acc[c + 4 * t + 2]);
          acc[c + 4 * t + 3] = fmaf(__uint_as_float(v[4 * t + 3]), f.w, acc[c + 4 * t + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar_tempty(buf));
        mbar_arrive(bar_sempty(r));
      }
    }
  }

  // ------------------------------------------------------------ teardown --
  const int n_loc = q * 32 + lane;  // epilogue thread's weight row inside the tile
  if (is_epi && S > 1 && *abort_flag == 0) {
    // fp32 partial tile, rows = tokens, 128 floats per row (coalesced 128 B per warp store)
    const int64_t tile = static_cast<int64_t>(mt) * gridDim.x + nt;
    float* part = p.partials + ((tile * S + s) * BN) * kTileW;
#pragma unroll
    for (int j = 0; j < C::kCpw; ++j) {
      const int row = col0 + j;
      if (m0 + row < p.M) __stcg(part + row * kTileW + n_loc, acc[j]);
    }
    __threadfence();
  }
  tc_fence_before();
  __syncthreads();  // every role has left its loop: the abort flag is final from here on
  tc_fence_after();
  const bool ok = (*abort_flag == 0);
  if (warp == 0) {
    // Producer: if the pipeline was abandoned, wait (bounded, fresh deadline)
    // for the TMA copies it issued so none lands after the CTA has exited.
    if (!ok && lane == 0) {
      const int first = produced > C::kStages ? produced - C::kStages : 0;
      volatile int no_abort = 0;
      for (int i = first; i < produced; ++i)
        wait_bounded(bar_full(i % C::kStages), (i / C::kStages) & 1, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
  } else if (warp == 1) {
    // No MMA may still be writing TMEM when it is freed: commit arrives once
    // every earlier tcgen05.mma of this thread has completed.
    if (lane == 0) {
      umma_commit(bar_drain);
      volatile int no_abort = 0;
      wait_bounded(bar_drain, 0, &no_abort, status, kStDrain, tmo);
    }
    __syncwarp();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }

  if (S == 1) {
    if (!ok) return;
    // Stage the bf16 tile in shared memory (the A ring is idle now: every TMA
    // copy was consumed and every MMA reading it has completed), then write
    // 16-byte vectors along rows of Y.
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffA);
    if (is_epi) {
#pragma unroll
      for (int j = 0; j < C::kCpw; ++j) stg[(col0 + j) * kTileW + n_loc] = __float2bfloat16_rn(acc[j]);
    }
    __syncthreads();
    const int rows = min(BN, p.M - m0);
    const int chunks = rows * (kTileW / 8);           // 16-byte chunks
    for (int c = threadIdx.x; c < chunks; c += kThreads) {
      const int row = c >> 4;
      const int cc = c & 15;
      const uint4 v = *reinterpret_cast<const uint4*>(stg + row * kTileW + cc * 8);
      *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(m0 + row) * p.ldo + n0 + cc * 8) = v;
    }
    return;
  }

  // Split-K: publish partials to the cluster (every CTA arrives, also after
  // an abort, so no CTA of the cluster waits forever), then reduce a disjoint
  // block of rows over the slices in fixed order.
  cluster_sync_all();
  if (!ok) return;
  const int64_t tile = static_cast<int64_t>(mt) * gridDim.x + nt;
  const float* part0 = p.partials + (tile * S) * BN * kTileW;
  const int rows = min(BN, p.M - m0);
  const int per = (rows + S - 1) / S;
  const int r0 = s * per;
  const int r1 = min(rows, r0 + per);
  const int items = (r1 > r0 ? r1 - r0 : 0) * (kTileW / 4);
  for (int it = threadIdx.x; it < items; it += kThreads) {
    const int row = r0 + (it >> 5);
    const int c4 = it & 31;
    const float* src = part0 + row * kTileW + c4 * 4;
    float4 sum = __ldcg(reinterpret_cast<const float4*>(src));
    for (int t = 1; t < S; ++t) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + static_cast<int64_t>(t) * BN * kTileW));
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(sum.x, sum.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(sum.z, sum.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p.out + static_cast<int64_t>(m0 + row) * p.ldo + n0 + c4 * 4) = pk;
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

struct DeviceInfo {
  bool init = false;
  bool sm100 = false;
  int sms = 0;
  unsigned configured = 0;  // bit per token-tile variant: dynamic smem attribute set
};

static std::mutex g_mu;
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

// Token tile for M: one tile up to 256 tokens, else the fewest 256-wide
// tiles, each rounded up to a multiple of 32.
static int pick_tile_m(int M) {
  const int tiles = (M + 255) / 256;
  const int per = (M + tiles - 1) / tiles;
  int bn = ((per + 31) / 32) * 32;
  return bn < 32 ? 32 : bn;
}

// Split-K choice: the stand-in for aiter's tuned (M,N,K,cu_num) table.  Cost
// model in units of one 128-wide K step of one CTA: waves * steps-per-CTA,
// plus a fixed cost per extra slice for writing and re-reading the fp32
// partial tile.  Slices keep >= 4 K steps each.
static int pick_split(int M, int N, int K, int bn, int sms) {
  const int KB = K / kBlk;
  const int tiles = (N / kTileW) * ((M + bn - 1) / bn);
  int best = 1;
  double best_cost = 1e30;
  for (int sp = 1; sp <= kMaxSplit; ++sp) {
    if (sp > 1 && KB / sp < 4) break;
    const int ctas = tiles * sp;
    const int waves = (ctas + sms - 1) / sms;
    const int steps = (KB + sp - 1) / sp;
    const double reduce = sp > 1 ? 2.0 + 4.0 * bn / 256.0 : 0.0;
    const double cost = static_cast<double>(waves) * steps + reduce;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

static size_t workspace_bytes_for(int M, int N, int bn, int split) {
  if (split <= 1) return 0;
  const size_t tiles = static_cast<size_t>(N / kTileW) * ((M + bn - 1) / bn);
  return tiles * split * bn * kTileW * sizeof(float);
}

static int encode_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FACK_OK : FACK_ERR_BAD_ALIGN;
}

template <int BN>
static int launch_bn(DeviceInfo* d, const CUtensorMap& tw, const CUtensorMap& tx, const Params& p, int M,
                     cudaStream_t stream) {
  using C = Cfg<BN>;
  auto kern = gemm_bs_kernel<BN>;
  const unsigned bit = 1u << (BN / 32 - 1);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!(d->configured & bit)) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
        return FACK_ERR_LAUNCH;
      d->configured |= bit;
    }
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(p.N / kTileW, (M + BN - 1) / BN, p.split);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (p.split > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = p.split;
    cfg.numAttrs = 1;
  }
  if (cudaLaunchKernelEx(&cfg, kern, tw, tx, p) != cudaSuccess) return FACK_ERR_LAUNCH;
  return FACK_OK;
}

static bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

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
    default: return "unknown status";
  }
}

int fack_version(void) { return 100; }

int fack_gemm_bs_select(int M, int N, int K, int split_k_request, int* tile_m, int* split_k) {
  if (M < 1 || N < kBlk || K < kBlk || N % kBlk || K % kBlk) return FACK_ERR_BAD_SHAPE;
  if (!tile_m || !split_k) return FACK_ERR_BAD_ARG;
  const int bn = pick_tile_m(M);
  const int KB = K / kBlk;
  int sp = split_k_request;
  if (sp < 0 || sp > kMaxSplit || sp > KB) return FACK_ERR_BAD_ARG;
  if (sp == 0) {
    DeviceInfo* d = nullptr;
    const int st = device_info(&d);
    if (st != FACK_OK) return st;
    sp = pick_split(M, N, K, bn, d->sms);
  }
  *tile_m = bn;
  *split_k = sp;
  return FACK_OK;
}

int fack_gemm_bs_workspace_size(int M, int N, int K, int split_k, size_t* bytes) {
  if (!bytes) return FACK_ERR_BAD_ARG;
  int bn = 0, sp = 0;
  const int st = fack_gemm_bs_select(M, N, K, split_k, &bn, &sp);
  if (st != FACK_OK) return st;
  *bytes = workspace_bytes_for(M, N, bn, sp);
  return FACK_OK;
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

int fack_gemm_bs(const void* xq, int64_t ldx, const void* wq, int wq_packed, const float* x_scale,
                 int64_t xs_stride_m, int64_t xs_stride_kb, const float* w_scale, void* out, int64_t ldo, int M,
                 int N, int K, int split_k, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 1 || N < kBlk || K < kBlk || N % kBlk || K % kBlk) return FACK_ERR_BAD_SHAPE;
  if (M > (1 << 24)) return FACK_ERR_BAD_SHAPE;
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
  const int bn = pick_tile_m(M);
  const int sp = split_k ? split_k : pick_split(M, N, K, bn, d->sms);
  const size_t need = workspace_bytes_for(M, N, bn, sp);
  if (need && (!workspace || workspace_bytes < need || !aligned(workspace, 16))) return FACK_ERR_WS_TOO_SMALL;

  CUtensorMap tw, tx;
  if (wq_packed == FACK_W_PACKED)
    st = encode_2d(&tw, wq, kBlk, static_cast<uint64_t>(N) * KB, kBlk, kBlk, kTileW,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    st = encode_2d(&tw, wq, K, N, K, kBlk, kTileW, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != FACK_OK) return st;
  st = encode_2d(&tx, xq, K, M, ldx, kBlk, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != FACK_OK) return st;

  Params p;
  p.x_scale = x_scale;
  p.xs_sm = xs_stride_m;
  p.xs_sk = xs_stride_kb;
  p.w_scale = w_scale;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.partials = static_cast<float*>(workspace);
  p.M = M;
  p.N = N;
  p.K = K;
  p.KB = KB;
  p.split = sp;
  p.w_packed = wq_packed;
  p.timeout_ns = 2000000000ull;  // 2 s: far above any legitimate wait, short enough to report a lost arrival

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (bn) {
    case 32: return launch_bn<32>(d, tw, tx, p, M, s);
    case 64: return launch_bn<64>(d, tw, tx, p, M, s);
    case 96: return launch_bn<96>(d, tw, tx, p, M, s);
    case 128: return launch_bn<128>(d, tw, tx, p, M, s);
    case 160: return launch_bn<160>(d, tw, tx, p, M, s);
    case 192: return launch_bn<192>(d, tw, tx, p, M, s);
    case 224: return launch_bn<224>(d, tw, tx, p, M, s);
    case 256: return launch_bn<256>(d, tw, tx, p, M, s);
    default: return FACK_ERR_BAD_ARG;
  }
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
