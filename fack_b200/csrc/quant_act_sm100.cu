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
// HBM-bound byte work: a warp owns one 128-element group at a time (4
// elements per lane, one 16 B or 8 B load), reduces the group's amax with
// shuffles, divides with IEEE division, converts with the hardware
// round-to-nearest-even e4m3 conversion and writes 4 codes per lane (128 B per
// warp).  Each warp streams its own contiguous run of groups with 4 (fp32) or
// 8 (bf16) groups in flight, so enough bytes are outstanding per SM to stream
// at HBM rate.

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fack_gemm.h"

namespace fack_quant {

constexpr int kBlk = 128;
constexpr float kQmax = 240.0f;
constexpr int kThreads = 256;

// Raw 4-element loads (kept as loaded until used, so the bytes in flight cost
// as few registers as possible) and their widening to fp32.
struct Raw4F32 {
  float4 r;
};
struct Raw4BF16 {
  uint2 r;
};
__device__ __forceinline__ void load_raw(const float* p, Raw4F32& v) {
  v.r = __ldcs(reinterpret_cast<const float4*>(p));  // streamed once
}
__device__ __forceinline__ void load_raw(const __nv_bfloat16* p, Raw4BF16& v) {
  v.r = __ldcs(reinterpret_cast<const uint2*>(p));
}
__device__ __forceinline__ void widen(const Raw4F32& v, float (&f)[4]) {
  f[0] = v.r.x;
  f[1] = v.r.y;
  f[2] = v.r.z;
  f[3] = v.r.w;
}
__device__ __forceinline__ void widen(const Raw4BF16& v, float (&f)[4]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.r.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.r.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}
template <typename T> struct RawOf;
template <> struct RawOf<float> { using type = Raw4F32; };
template <> struct RawOf<__nv_bfloat16> { using type = Raw4BF16; };

__device__ __forceinline__ uint32_t quant4(const float (&v)[4], float scale) {
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float q = fminf(fmaxf(v[i] / scale, -kQmax), kQmax);
    const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3);
    packed |= static_cast<uint32_t>(b) << (8 * i);
  }
  return packed;
}

// Groups in flight per warp: ~2 KB of input per warp keeps enough bytes
// outstanding per SM to stream at HBM rate.
template <typename T>
struct InFlight {
  static constexpr int value = 2048 / (kBlk * static_cast<int>(sizeof(T)));
};

template <typename T>
__global__ void __launch_bounds__(kThreads) quant_act_kernel(const T* __restrict__ x, int64_t ldx, int M, int KB,
                                                             uint8_t* __restrict__ xq, int64_t ldq,
                                                             float* __restrict__ xs, int64_t xs_sm,
                                                             int64_t xs_sk) {
  constexpr int U = InFlight<T>::value;
  using Raw = typename RawOf<T>::type;
  const int lane = threadIdx.x & 31;
  const int64_t groups = static_cast<int64_t>(M) * KB;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  // each warp owns a contiguous run of groups (row-major over (m, kb)), so it
  // streams one contiguous stretch of X and of the codes; (m, kb) advance by
  // increments, with no division in the loop
  const int64_t g_begin = w * groups / nwarps;
  const int64_t g_end = (w + 1) * groups / nwarps;
  int64_t m = g_begin / KB;
  int kb = static_cast<int>(g_begin - m * KB);
  for (int64_t g0 = g_begin; g0 < g_end; g0 += U) {
    Raw raw[U];
    const int64_t m0 = m;
    const int kb0 = kb;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (g0 + u < g_end) load_raw(x + m * ldx + kb * kBlk + lane * 4, raw[u]);
      if (++kb == KB) {
        kb = 0;
        ++m;
      }
    }
    int64_t mu = m0;
    int ku = kb0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (g0 + u >= g_end) break;  // warp-uniform
      float v[4];
      widen(raw[u], v);
      float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      const float scale = a > 0.0f ? a / kQmax : 1.0f;
      *reinterpret_cast<uint32_t*>(xq + mu * ldq + ku * kBlk + lane * 4) = quant4(v, scale);
      if (lane == 0) xs[mu * xs_sm + ku * xs_sk] = scale;
      if (++ku == KB) {
        ku = 0;
        ++mu;
      }
    }
  }
}

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

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
  const int KB = K / kBlk;
  const int64_t groups = static_cast<int64_t>(M) * KB;
  // one resident wave of the grid-stride loop (occupancy of the variant),
  // never more warps than groups
  static int resident[2] = {0, 0};
  int& per_sm = resident[x_dtype];
  if (per_sm == 0) {
    const cudaError_t e =
        x_dtype == FACK_DTYPE_F32
            ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quant_act_kernel<float>, kThreads, 0)
            : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quant_act_kernel<__nv_bfloat16>, kThreads, 0);
    if (e != cudaSuccess || per_sm < 1) return FACK_ERR_CUDA;
  }
  const int64_t want = (groups + (kThreads / 32) * 8 - 1) / ((kThreads / 32) * 8);  // >= 8 groups per warp
  const int64_t wave = static_cast<int64_t>(sms) * per_sm;
  const int blocks = static_cast<int>(want < wave ? want : wave);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == FACK_DTYPE_F32)
    quant_act_kernel<float><<<blocks, kThreads, 0, s>>>(static_cast<const float*>(x), ldx, M, KB,
                                                         static_cast<uint8_t*>(xq), ldq, x_scale, xs_stride_m,
                                                         xs_stride_kb);
  else
    quant_act_kernel<__nv_bfloat16><<<blocks, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, M, KB,
                                                                 static_cast<uint8_t*>(xq), ldq, x_scale,
                                                                 xs_stride_m, xs_stride_kb);
  return cudaGetLastError() == cudaSuccess ? FACK_OK : FACK_ERR_LAUNCH;
}
