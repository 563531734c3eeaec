// tuned_table.h -- internal interface of the exact-shape plan tables
// (tuned_table.cpp) used by the GEMM planners (gemm_bs_sm100.cu,
// gemm_tn_sm100.cu).
#pragma once

#include <string>

#include "fack_internal.h"

namespace fack {

constexpr int kTunedMaxSplit = 8;  // the GEMM's cluster limit along K

// Checks a fully specified plan against the kernel's rules: M >= 1, N and K
// positive multiples of 128; tile_m 128 (one CTA) or 256 (a CTA pair) with
// tile_n 64, 128 or 256 dividing N, 1 <= split_k <= min(8, K/128), and
// 2 * split_k <= 8 for a pair; or tile_m 16, 32, 64 (swapped small-M tiles,
// M <= tile_m) with tile_n 128 and at most 128 K blocks per slice.  Returns a
// FACK_* status.
int tuned_validate(int M, int N, int K, int tile_m, int tile_n, int split_k);

// The FP8 table's row for (cu_num, M, N, K), if any.  Thread-safe.
bool tuned_lookup(int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k);

// The sibling table's row for (kind = FACK_GEMM_BF16 | FACK_GEMM_I8, cu_num,
// M, N, K), if any.  Thread-safe.
bool tn_tuned_lookup(int kind, int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k);

// fack_bs_sm100_t<tile_m>x<tile_n>_s<split> in its canonical spelling.
bool parse_kernel_name(const std::string& name, int* tm, int* bn, int* sp);

}  // namespace fack
