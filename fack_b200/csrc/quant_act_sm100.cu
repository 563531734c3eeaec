// quant_act_sm100.cu -- fused activation quantisation feeding the FP8 GEMM (sm_100a).
//
// One pass over X (fp32 or bf16, [M, K] row-major) produces the GEMM's inputs:
//   x_scale[m, kb] = amax(|x[m, kb*128 : kb*128+128]|) / 240   (1 for an all-zero group)
//   xq[m, k]       = e4m3fn(clamp(x[m, k] / x_scale[m, k/128], -240, 240))
// the construction of the benchmark inputs (scale = amax/240; every code is
// then exactly representable in e4m3fn and in the reference's e4m3fnuz), with
// x_scale written straight into the caller's layout -- e.g. the reference's
// transposed-contiguous view (client/aiter/hsa/gfx942/driver.py:22:
// sa.T.contiguous().view_as(sa), i.e. stride_m = 1, stride_kb = M).
//
// HBM-bound byte work, staged through shared memory: two persistent CTAs per
// SM; in each, one thread streams row chunks (up to 32 groups of 128 elements,
// <= 16 KB) with 1-D bulk copies into a 4-stage ring, so the bytes in flight sit in
// shared memory rather than registers; sixteen warps each take two groups at
// a time from the landed chunk (4 elements per lane), reduce its amax with
// one warp-wide integer max (redux.sync) on the magnitudes' bit patterns,
// divide with IEEE division, convert with the hardware round-to-nearest-even
// e4m3 conversion and store 4 codes per lane (128 B per warp).  Every mbarrier wait is bounded; on expiry the CTA records a flag in
// the library's device status word, drains its copies and exits.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/fack_gemm.h"
#include "fack_internal.h"
#include "sm100_ptx.cuh"


namespace fack_quant {

using namespace fack;

constexpr int kBlk = 128;
constexpr float kQmax = 240.0f;

constexpr int kStages = 4;
constexpr int kChunkGroups = 32;                 // groups of 128 elements per chunk (one row segment)
constexpr int kConsumerWarps = 16;
constexpr int kQThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr unsigned kStQuant = 64u;               // status flag: a wait in the quantiser gave up

// clamp(v / scale) to +-240 (IEEE division) and convert to e4m3 (round to
// nearest even), two values per conversion; 4 codes packed little-endian
__device__ __forceinline__ uint32_t quant4(const float (&v)[4], float scale) {
  float q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = fminf(fmaxf(v[i] / scale, -kQmax), kQmax);
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(q[0], q[1]), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(q[2], q[3]), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

__device__ __forceinline__ void lds4(uint32_t addr, const float*, float (&v)[4]) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]) : "r"(addr));
}
__device__ __forceinline__ void lds4(uint32_t addr, const __nv_bfloat16*, float (&v)[4]) {
  uint32_t lo, hi;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(lo), "=r"(hi) : "r"(addr));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lo));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hi));
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}

template <typename T>
__global__ void __launch_bounds__(kQThreads, 2) quant_act_kernel(const T* __restrict__ x, int64_t ldx, int M, int KB,
                                                                 uint8_t* __restrict__ xq, int64_t ldq,
                                                                 float* __restrict__ xs, int64_t xs_sm,
                                                                 int64_t xs_sk, unsigned int* status,
                                                                 uint64_t timeout_ns) {
  constexpr int kChunkBytes = kChunkGroups * kBlk * static_cast<int>(sizeof(T));
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ int abort_flag_s;
  volatile int* abort_flag = &abort_flag_s;
  const uint32_t ring = smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_row = (KB + kChunkGroups - 1) / kChunkGroups;     // chunks per row
  const int64_t chunks = static_cast<int64_t>(M) * per_row;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), kConsumerWarps);
    }
    abort_flag_s = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int64_t issued = 0;
      for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x, ++issued) {
        const int st = static_cast<int>(issued % kStages);
        const uint32_t ph = static_cast<uint32_t>(issued / kStages) & 1u;
        if (!wait_bounded(smem_addr(&empty[st]), ph ^ 1u, abort_flag, status, kStQuant, timeout_ns)) break;
        const int64_t m = c / per_row;
        const int g0 = static_cast<int>(c - m * per_row) * kChunkGroups;
        const int ng = KB - g0 < kChunkGroups ? KB - g0 : kChunkGroups;
        const uint32_t bytes = static_cast<uint32_t>(ng) * kBlk * sizeof(T);
        mbar_arrive_expect_tx(smem_addr(&full[st]), bytes);
        bulk_load_1d(ring + st * kChunkBytes, x + m * ldx + static_cast<int64_t>(g0) * kBlk, bytes,
                     smem_addr(&full[st]));
      }
      if (*abort_flag) {
        // no copy may land after the CTA exits: wait (bounded, fresh deadline)
        // for the last stages issued
        volatile int no_abort = 0;
        const int64_t first = issued > kStages ? issued - kStages : 0;
        for (int64_t i = first; i < issued; ++i)
          wait_bounded(smem_addr(&full[i % kStages]), static_cast<uint32_t>(i / kStages) & 1u, &no_abort, status,
                       kStQuant, timeout_ns);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers --
    int64_t used = 0;
    for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x, ++used) {
      const int st = static_cast<int>(used % kStages);
      const uint32_t ph = static_cast<uint32_t>(used / kStages) & 1u;
      const bool got = wait_bounded(smem_addr(&full[st]), ph, abort_flag, status, kStQuant, timeout_ns);
      if (!__all_sync(0xffffffffu, got)) break;
      const int64_t m = c / per_row;
      const int g0 = static_cast<int>(c - m * per_row) * kChunkGroups;
      const int ng = KB - g0 < kChunkGroups ? KB - g0 : kChunkGroups;
      // two groups per warp at a time (j and j + kConsumerWarps), interleaved
      // so their dependent reduce / divide / convert chains overlap
      for (int j = warp; j < ng; j += 2 * kConsumerWarps) {
        const bool two = j + kConsumerWarps < ng;  // warp-uniform
        float v[2][4];
        lds4(ring + st * kChunkBytes + (j * kBlk + lane * 4) * static_cast<int>(sizeof(T)),
             static_cast<const T*>(nullptr), v[0]);
        if (two)
          lds4(ring + st * kChunkBytes + ((j + kConsumerWarps) * kBlk + lane * 4) * static_cast<int>(sizeof(T)),
               static_cast<const T*>(nullptr), v[1]);
        float a[2];
#pragma unroll
        for (int u = 0; u < 2; ++u)
          a[u] = fmaxf(fmaxf(fabsf(v[u][0]), fabsf(v[u][1])), fmaxf(fabsf(v[u][2]), fabsf(v[u][3])));
        // warp maximum in one instruction each: for non-negative floats the bit
        // patterns order as unsigned integers
        a[0] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(a[0])));
        a[1] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(a[1])));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (u == 1 && !two) break;
          const float scale = a[u] > 0.0f ? a[u] / kQmax : 1.0f;
          const int64_t kb = g0 + j + u * kConsumerWarps;
          *reinterpret_cast<uint32_t*>(xq + m * ldq + kb * kBlk + lane * 4) = quant4(v[u], scale);
          if (lane == 0) xs[m * xs_sm + kb * xs_sk] = scale;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&empty[st]));
    }
  }
  __syncthreads();
}

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Kernel attributes are set per device: one bit per (device, input type).
constexpr int kMaxDevices = 64;
static std::mutex g_configure_mu;
static uint32_t g_configured[kMaxDevices];

static bool configure_once(int dev, int bit, const void* fn, int smem) {
  if (dev < 0 || dev >= kMaxDevices) return false;
  std::lock_guard<std::mutex> lk(g_configure_mu);
  if (g_configured[dev] & (1u << bit)) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return false;
  g_configured[dev] |= 1u << bit;
  return true;
}

}  // namespace fack_quant

extern "C" int fack_quant_act(const void* x, int x_dtype, int64_t ldx, int M, int K, void* xq, int64_t ldq,
                              float* x_scale, int64_t xs_stride_m, int64_t xs_stride_kb, void* stream) {
  using namespace fack_quant;
  if (M < 1 || K < kBlk || K % kBlk || M > (1 << 24)) return FACK_ERR_BAD_SHAPE;
  if (x_dtype != FACK_DTYPE_F32 && x_dtype != FACK_DTYPE_BF16) return FACK_ERR_BAD_ARG;
  if (!x || !xq || !x_scale) return FACK_ERR_BAD_ALIGN;
  if (!aligned(x, 16) || !aligned(xq, 16) || !aligned(x_scale, 4)) return FACK_ERR_BAD_ALIGN;
  if (ldx < K || ldx % 8 || ldq < K || ldq % 16 || xs_stride_m < 1 || xs_stride_kb < 1) return FACK_ERR_BAD_STRIDE;
  int dev = 0, major = 0, minor = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return FACK_ERR_CUDA;
  if (major != 10 || minor != 0) return FACK_ERR_UNSUPPORTED_ARCH;
  unsigned int* status = fack::device_status_word();
  if (!status) return FACK_ERR_CUDA;
  const int KB = K / kBlk;
  const int64_t chunks = static_cast<int64_t>(M) * ((KB + kChunkGroups - 1) / kChunkGroups);
  // two persistent CTAs per SM (32 quantising warps), never more CTAs than chunks
  const int blocks = static_cast<int>(chunks < 2 * sms ? chunks : 2 * sms);
  const int smem_f32 = kStages * kChunkGroups * kBlk * 4, smem_bf16 = kStages * kChunkGroups * kBlk * 2;
  const uint64_t tmo = 2000000000ull;  // 2 s
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == FACK_DTYPE_F32) {
    if (!configure_once(dev, 0, reinterpret_cast<const void*>(quant_act_kernel<float>), smem_f32))
      return FACK_ERR_LAUNCH;
    quant_act_kernel<float><<<blocks, kQThreads, smem_f32, s>>>(static_cast<const float*>(x), ldx, M, KB,
                                                                 static_cast<uint8_t*>(xq), ldq, x_scale, xs_stride_m,
                                                                 xs_stride_kb, status, tmo);
  } else {
    if (!configure_once(dev, 1, reinterpret_cast<const void*>(quant_act_kernel<__nv_bfloat16>), smem_bf16))
      return FACK_ERR_LAUNCH;
    quant_act_kernel<__nv_bfloat16><<<blocks, kQThreads, smem_bf16, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, M, KB, static_cast<uint8_t*>(xq), ldq, x_scale, xs_stride_m,
        xs_stride_kb, status, tmo);
  }
  return cudaGetLastError() == cudaSuccess ? FACK_OK : FACK_ERR_LAUNCH;
}
