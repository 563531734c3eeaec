// fack_internal.h -- host-side helpers shared by the library's translation
// units (defined in gemm_bs_sm100.cu).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace fack {

// Records `what` as the calling thread's fack_last_error text and returns
// `status`.
int record_error(int status, const char* what);

// Current device: FACK_OK with its SM count when it is an sm_100 part (and the
// tensor-map encoder is available), else FACK_ERR_UNSUPPORTED_ARCH /
// FACK_ERR_CUDA.
int sm100_device(int* sms);

// 2-D byte tensor map: `outer` rows of `inner` bytes, rows `row_bytes` apart,
// box of box_inner bytes x box_outer rows, 128-byte swizzle or none.
// FACK_ERR_BAD_ALIGN if the driver refuses the layout.
int encode_bytes_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// Device address of the library's status word on the current device (NULL
// on failure); kernels OR a flag into it when a bounded wait gives up.
unsigned int* device_status_word();

}  // namespace fack
