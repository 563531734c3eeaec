// tuned_table.cpp -- exact-shape (tile, split-K) overrides for the GEMM
// planners: the FP8 block-scaled GEMM (fack_gemm_bs_plan) and the sibling
// BF16 / INT8 families (fack_gemm_tn_plan).
//
// The reference picks its kernel by an exact (cu_num, M, N, K) row of a tuned
// CSV (client/aiter/dispatch.py:23-35 names the blockscale-preshuffle table
// and its key columns "M N K"; rows carry kernelName and splitK, and a row
// reporting a non-zero error ratio is refused, dispatch.py:135-137).  This
// file holds the B200 counterpart: one table keyed by (family, SM count, M, N,
// K) whose rows fix the token tile, weight tile and split-K of a planner's
// fully automatic choice.  Shapes without a row keep the cost-model plan.
//
// CSV form read by fack_gemm_bs_tuned_load / fack_gemm_tn_tuned_load: '#'
// lines are comments; the first other line is a header; columns are found by
// name, so order and extra columns do not matter.  Required: cu_num, M, N, K,
// kernelName -- for the FP8 table this library's
// fack_bs_sm100_t{16|32|64|128|256}x{64|128|224|256}_s{S}, for the sibling table
// fack_tn_sm100_{bf16|i8}_t{128|256}x{64|128|256}_s{S} (the name gives the
// family).  Optional: splitK (must equal the name's S) and errRatio (must be
// 0).  Rows naming another kernel family (a gfx942 symbol, or the other table's
// names) are skipped and counted; a name with the table's own prefix that is
// not in the canonical form is an error.  The file is checked whole before any
// row is added: a bad row leaves the table as it was.

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <fstream>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/fack_gemm.h"
#include "tuned_table.h"

namespace fack {
namespace {

// Family of a row: the FP8 block-scaled GEMM, or a sibling kind
// (FACK_GEMM_BF16 / FACK_GEMM_I8).
constexpr int kFamilyBlockscale = 100;

using Key = std::tuple<int, int, int, int, int>;  // family, cu_num, M, N, K

struct Plan {
  int tile_m, tile_n, split_k;
};

std::mutex g_mu;
std::map<Key, Plan> g_rows;

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && (s[a] == ' ' || s[a] == '\t' || s[a] == '"' || s[a] == '\r')) ++a;
  while (b > a && (s[b - 1] == ' ' || s[b - 1] == '\t' || s[b - 1] == '"' || s[b - 1] == '\r')) --b;
  return s.substr(a, b - a);
}

std::vector<std::string> split_csv(const std::string& line) {
  std::vector<std::string> out;
  std::string cur;
  for (char c : line) {
    if (c == ',') {
      out.push_back(trim(cur));
      cur.clear();
    } else {
      cur.push_back(c);
    }
  }
  out.push_back(trim(cur));
  return out;
}

bool parse_int(const std::string& s, int* v) {
  if (s.empty()) return false;
  char* end = nullptr;
  const long x = strtol(s.c_str(), &end, 10);
  if (*end != '\0' || x < -2147483647L || x > 2147483647L) return false;
  *v = static_cast<int>(x);
  return true;
}

bool parse_double(const std::string& s, double* v) {
  if (s.empty()) return false;
  char* end = nullptr;
  *v = strtod(s.c_str(), &end);
  return *end == '\0';
}

int bad_row(const char* path, int line, const char* why) {
  char msg[256];
  snprintf(msg, sizeof(msg), "%s:%d: %s", path, line, why);
  return record_error(FACK_ERR_BAD_ARG, msg);
}

// fack_tn_sm100_<bf16|i8>_t<tile_m>x<tile_n>_s<split>, canonical spelling only.
bool parse_tn_name(const std::string& name, int* kind, int* tm, int* bn, int* sp) {
  char fam[8] = {0};
  int n = -1;
  if (sscanf(name.c_str(), "fack_tn_sm100_%7[a-z0-9]_t%dx%d_s%d%n", fam, tm, bn, sp, &n) != 4) return false;
  if (n != static_cast<int>(name.size())) return false;
  if (strcmp(fam, "bf16") == 0) {
    *kind = FACK_GEMM_BF16;
  } else if (strcmp(fam, "i8") == 0) {
    *kind = FACK_GEMM_I8;
  } else {
    return false;
  }
  char canon[64];
  snprintf(canon, sizeof(canon), "fack_tn_sm100_%s_t%dx%d_s%d", fam, *tm, *bn, *sp);
  return name == canon;
}

// A fully specified sibling plan checked by the sibling planner's own rules
// (with all three given it answers without a device query).
int tn_validate(int kind, int M, int N, int K, int tm, int bn, int sp) {
  if (tm == 0 || bn == 0 || sp == 0) return FACK_ERR_BAD_ARG;
  int a, b, c;
  return fack_gemm_tn_plan(kind, M, N, K, tm, bn, sp, &a, &b, &c);
}

// Which kernel names a table reads, and how a row is checked.
struct TableKind {
  const char* prefix;  // names with this prefix belong to the table (malformed ones are errors)
  bool (*parse)(const std::string& name, int* family, int* tm, int* bn, int* sp);
  int (*validate)(int family, int M, int N, int K, int tm, int bn, int sp);
};

bool parse_bs_row_name(const std::string& name, int* family, int* tm, int* bn, int* sp) {
  *family = kFamilyBlockscale;
  return parse_kernel_name(name, tm, bn, sp);
}

int validate_bs_row(int, int M, int N, int K, int tm, int bn, int sp) { return tuned_validate(M, N, K, tm, bn, sp); }

const TableKind kBlockscaleTable = {"fack_bs_sm100_", parse_bs_row_name, validate_bs_row};
const TableKind kSiblingTable = {"fack_tn_sm100_", parse_tn_name, tn_validate};

int load_csv(const char* path, const TableKind& table, int* rows_loaded, int* rows_skipped) {
  if (!path) return FACK_ERR_BAD_ARG;
  std::ifstream in(path);
  if (!in) return record_error(FACK_ERR_BAD_ARG, "tuned table: cannot open file");
  std::string line;
  std::vector<std::string> header;
  int c_cu = -1, c_m = -1, c_n = -1, c_k = -1, c_name = -1, c_split = -1, c_err = -1;
  std::vector<std::pair<Key, Plan>> rows;
  int skipped = 0, lineno = 0;
  while (std::getline(in, line)) {
    ++lineno;
    const std::string t = trim(line);
    if (t.empty() || t[0] == '#') continue;
    const std::vector<std::string> f = split_csv(line);
    if (header.empty()) {
      header = f;
      for (int i = 0; i < static_cast<int>(f.size()); ++i) {
        if (f[i] == "cu_num") c_cu = i;
        else if (f[i] == "M") c_m = i;
        else if (f[i] == "N") c_n = i;
        else if (f[i] == "K") c_k = i;
        else if (f[i] == "kernelName") c_name = i;
        else if (f[i] == "splitK") c_split = i;
        else if (f[i] == "errRatio" || f[i] == "err_ratio") c_err = i;
      }
      if (c_cu < 0 || c_m < 0 || c_n < 0 || c_k < 0 || c_name < 0)
        return bad_row(path, lineno, "header lacks one of cu_num, M, N, K, kernelName");
      continue;
    }
    if (f.size() != header.size()) return bad_row(path, lineno, "field count differs from the header");
    int cu, M, N, K;
    if (!parse_int(f[c_cu], &cu) || !parse_int(f[c_m], &M) || !parse_int(f[c_n], &N) || !parse_int(f[c_k], &K))
      return bad_row(path, lineno, "cu_num, M, N, K must be integers");
    int fam, tm, bn, sp;
    if (!table.parse(f[c_name], &fam, &tm, &bn, &sp)) {
      if (f[c_name].rfind(table.prefix, 0) == 0) {
        char why[96];
        snprintf(why, sizeof(why), "malformed %.20s kernelName", table.prefix);
        return bad_row(path, lineno, why);
      }
      ++skipped;  // another kernel family's row
      continue;
    }
    if (cu < 1) return bad_row(path, lineno, "cu_num must be >= 1");
    if (table.validate(fam, M, N, K, tm, bn, sp) != FACK_OK)
      return bad_row(path, lineno, "kernelName's tile or split is invalid for this shape");
    if (c_split >= 0) {
      int s2;
      if (!parse_int(f[c_split], &s2) || s2 != sp) return bad_row(path, lineno, "splitK disagrees with kernelName");
    }
    if (c_err >= 0 && !f[c_err].empty()) {
      double e;
      if (!parse_double(f[c_err], &e) || e != 0.0) return bad_row(path, lineno, "row reports a non-zero errRatio");
    }
    rows.emplace_back(Key(fam, cu, M, N, K), Plan{tm, bn, sp});
  }
  if (header.empty()) return record_error(FACK_ERR_BAD_ARG, "tuned table: no header line");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (const auto& r : rows) g_rows[r.first] = r.second;  // a later row for the same key wins
  }
  if (rows_loaded) *rows_loaded = static_cast<int>(rows.size());
  if (rows_skipped) *rows_skipped = skipped;
  return FACK_OK;
}

bool is_sibling(int family) { return family == FACK_GEMM_BF16 || family == FACK_GEMM_I8; }

int count_rows(bool sibling) {
  std::lock_guard<std::mutex> lk(g_mu);
  int n = 0;
  for (const auto& r : g_rows) n += is_sibling(std::get<0>(r.first)) == sibling;
  return n;
}

void clear_rows(bool sibling) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto it = g_rows.begin(); it != g_rows.end();) {
    if (is_sibling(std::get<0>(it->first)) == sibling)
      it = g_rows.erase(it);
    else
      ++it;
  }
}

bool lookup(int family, int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k) {
  std::lock_guard<std::mutex> lk(g_mu);
  const auto it = g_rows.find(Key(family, cu_num, M, N, K));
  if (it == g_rows.end()) return false;
  *tile_m = it->second.tile_m;
  *tile_n = it->second.tile_n;
  *split_k = it->second.split_k;
  return true;
}

}  // namespace

// fack_bs_sm100_t<tile_m>x<tile_n>_s<split>, nothing before or after, in the
// canonical spelling only (no sign, space or leading zero), as the Python
// layer's parser accepts it.
bool parse_kernel_name(const std::string& name, int* tm, int* bn, int* sp) {
  int n = -1;
  if (sscanf(name.c_str(), "fack_bs_sm100_t%dx%d_s%d%n", tm, bn, sp, &n) != 3) return false;
  if (n != static_cast<int>(name.size())) return false;
  char canon[64];
  snprintf(canon, sizeof(canon), "fack_bs_sm100_t%dx%d_s%d", *tm, *bn, *sp);
  return name == canon;
}

int tuned_validate(int M, int N, int K, int tile_m, int tile_n, int split_k) {
  if (M < 1 || N < 128 || K < 128 || N % 128 || K % 128 || M > 65535 * 128) return FACK_ERR_BAD_SHAPE;
  if (tile_n == 16) {  // warp-MMA small-M kernel: 16 weight rows, up to 16 tokens, no K split
    if (tile_m != 16 || M > tile_m || split_k != 1 || K / 128 > 256) return FACK_ERR_BAD_ARG;
    return FACK_OK;
  }
  if (tile_m == 16 || tile_m == 32 || tile_m == 64) {  // swapped small-M tiles: 128 weight rows, all M tokens
    if (M > tile_m || tile_n != 128 || split_k < 1 || split_k > kTunedMaxSplit || split_k > K / 128 ||
        (K / 128 + split_k - 1) / split_k > 128)
      return FACK_ERR_BAD_ARG;
    return FACK_OK;
  }
  if (tile_m != 128 && tile_m != 256) return FACK_ERR_BAD_ARG;
  if ((tile_n != 64 && tile_n != 128 && tile_n != 224 && tile_n != 256) || N % tile_n) return FACK_ERR_BAD_ARG;
  if (tile_n == 224 && (tile_m != 128 || split_k != 1)) return FACK_ERR_BAD_ARG;  // persistent kernel only
  if (split_k < 1 || split_k > kTunedMaxSplit || split_k > K / 128) return FACK_ERR_BAD_ARG;
  if (tile_m == 256 && 2 * split_k > kTunedMaxSplit) return FACK_ERR_BAD_ARG;
  return FACK_OK;
}

bool tuned_lookup(int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k) {
  return lookup(kFamilyBlockscale, cu_num, M, N, K, tile_m, tile_n, split_k);
}

bool tn_tuned_lookup(int kind, int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k) {
  return is_sibling(kind) && lookup(kind, cu_num, M, N, K, tile_m, tile_n, split_k);
}

}  // namespace fack

using namespace fack;

extern "C" {

int fack_gemm_bs_tuned_set(int cu_num, int M, int N, int K, int tile_m, int tile_n, int split_k) {
  if (cu_num < 1) return FACK_ERR_BAD_ARG;
  const int st = tuned_validate(M, N, K, tile_m, tile_n, split_k);
  if (st != FACK_OK) return st;
  std::lock_guard<std::mutex> lk(g_mu);
  g_rows[Key(kFamilyBlockscale, cu_num, M, N, K)] = Plan{tile_m, tile_n, split_k};
  return FACK_OK;
}

int fack_gemm_bs_tuned_lookup(int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k) {
  if (!tile_m || !tile_n || !split_k) return FACK_ERR_BAD_ARG;
  if (!tuned_lookup(cu_num, M, N, K, tile_m, tile_n, split_k)) *tile_m = *tile_n = *split_k = 0;
  return FACK_OK;
}

int fack_gemm_bs_tuned_count(void) { return count_rows(false); }

int fack_gemm_bs_tuned_clear(void) {
  clear_rows(false);
  return FACK_OK;
}

int fack_gemm_bs_tuned_load(const char* path, int* rows_loaded, int* rows_skipped) {
  return load_csv(path, kBlockscaleTable, rows_loaded, rows_skipped);
}

int fack_gemm_tn_tuned_set(int kind, int cu_num, int M, int N, int K, int tile_m, int tile_n, int split_k) {
  if (!is_sibling(kind) || cu_num < 1) return FACK_ERR_BAD_ARG;
  const int st = tn_validate(kind, M, N, K, tile_m, tile_n, split_k);
  if (st != FACK_OK) return st;
  std::lock_guard<std::mutex> lk(g_mu);
  g_rows[Key(kind, cu_num, M, N, K)] = Plan{tile_m, tile_n, split_k};
  return FACK_OK;
}

int fack_gemm_tn_tuned_lookup(int kind, int cu_num, int M, int N, int K, int* tile_m, int* tile_n, int* split_k) {
  if (!tile_m || !tile_n || !split_k || !is_sibling(kind)) return FACK_ERR_BAD_ARG;
  if (!tn_tuned_lookup(kind, cu_num, M, N, K, tile_m, tile_n, split_k)) *tile_m = *tile_n = *split_k = 0;
  return FACK_OK;
}

int fack_gemm_tn_tuned_count(void) { return count_rows(true); }

int fack_gemm_tn_tuned_clear(void) {
  clear_rows(true);
  return FACK_OK;
}

int fack_gemm_tn_tuned_load(const char* path, int* rows_loaded, int* rows_skipped) {
  return load_csv(path, kSiblingTable, rows_loaded, rows_skipped);
}

}  // extern "C"
