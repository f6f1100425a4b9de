// Host-side description of GGML formats and of the engine's device layout.
#pragma once
#include <stdint.h>

#include <string>

namespace qc {

// Reference quant.rs:5-11: (elements per block, bytes per block); false for unknown kinds.
inline bool ggml_block(uint32_t kind, uint64_t* elems, uint64_t* bytes) {
  switch (kind) {
    case 0: *elems = 1; *bytes = 4; return true;
    case 1: *elems = 1; *bytes = 2; return true;
    case 2: *elems = 32; *bytes = 18; return true;
    case 8: *elems = 32; *bytes = 34; return true;
    case 12: *elems = 256; *bytes = 144; return true;
    case 13: *elems = 256; *bytes = 176; return true;
    case 14: *elems = 256; *bytes = 210; return true;
  }
  return false;
}

// Reference quant.rs:12-21.  Returns 0 on success, or an error message.
inline const char* ggml_row_bytes(uint32_t kind, uint64_t cols, uint64_t* out) {
  uint64_t e, b;
  if (!ggml_block(kind, &e, &b)) return "GGML tensor type is not supported (supported: F32/F16/Q4_0/Q8_0/Q4_K/Q5_K/Q6_K)";
  if (cols == 0 || cols % e) return "row width is not divisible by block size";
  *out = cols / e * b;
  return nullptr;
}

// Device layout of a (rows x cols) matrix of `kind` (see MatDesc in common.cuh).
// Rows are stored in groups of 8: [8 rows of blocks][8 rows of d values], so a
// run of whole groups is one contiguous 16-byte-aligned span (8 * main_bytes and
// 8 * d_bytes are multiples of 16 for every kind).  Row counts are padded to a
// multiple of 8 with zero rows.
struct DevLayout {
  uint64_t main_bytes = 0;   // block bytes of one row (multiple of 16)
  uint64_t d_bytes = 0;      // d bytes of one row (0: no d values)
  uint64_t group_bytes = 0;  // 8 * (main_bytes + d_bytes)
  uint32_t units = 0, lpr = 1, upl = 1;
  uint64_t expert_bytes(uint64_t rows) const { return (rows + 7) / 8 * group_bytes; }
};

// Every row is processed in units of 64 elements: units = ceil(cols / 64).
inline DevLayout dev_layout(uint32_t kind, uint64_t cols) {
  DevLayout l;
  const uint64_t units = (cols + 63) / 64;
  l.units = (uint32_t)units;
  switch (kind) {
    case 12: l.main_bytes = cols / 256 * 144; break;
    case 13: l.main_bytes = cols / 256 * 176; break;
    case 14: l.main_bytes = cols / 256 * 208; l.d_bytes = cols / 256 * 2; break;
    case 8: l.main_bytes = units * 64; l.d_bytes = units * 4; break;  // two 32-blocks per unit
    case 2: l.main_bytes = units * 32; l.d_bytes = units * 4; break;
    case 1: l.main_bytes = units * 128; break;
    default: l.main_bytes = units * 256; break;
  }
  l.group_bytes = 8 * (l.main_bytes + l.d_bytes);
  uint32_t lpr = 1;
  while (lpr < 32 && l.units % (lpr * 2) == 0) lpr *= 2;
  l.lpr = lpr;
  l.upl = l.units / lpr;
  return l;
}

}  // namespace qc
