// Host-side RoPE (cos, sin) table, bit-identical to the values the reference
// computes inline in src/ops.cc:26-31 (normal) and :45-50 (NeoX).
//
// The reference evaluates, per pair j of a head at position p,
//   angle = (float)p / std::pow(theta, (float)(2j) / (float)hd)
// (NeoX writes the exponent as 2.0f * (float)j / (float)hd — the same float,
// since 2j is exact), then std::cos(angle) and std::sin(angle).  The float
// overloads of std::pow/cos/sin are powf/cosf/sinf, so this file calls those
// directly; it is compiled with -ffp-contract=off and without fast-math.
// Building the table on the host is what makes device RoPE exact: one ulp in
// the angle at position 16383 moves cos by ~4e-4.
#include <cmath>
#include <cstdint>

#include "mlb_ops.h"

extern "C" int mlb_rope_table_build_host(float theta, int hd,
                                         int64_t pos_begin, int64_t pos_end,
                                         float* out_host) {
  if (out_host == nullptr || hd <= 0 || (hd % 2) != 0 || pos_begin < 0 ||
      pos_end < pos_begin || !(theta > 0.0f)) {
    return MLB_ERR_ARG;
  }
  const int half = hd / 2;
  // The exponent's reciprocal power depends only on j: compute it once per j
  // (the same powf call the reference makes for every position).
  float denom[4096];
  float* den = denom;
  float* heap = nullptr;
  if (half > 4096) {
    heap = new float[half];
    den = heap;
  }
  for (int j = 0; j < half; ++j) {
    const float exponent =
        static_cast<float>(2 * j) / static_cast<float>(hd);
    den[j] = powf(theta, exponent);
  }
  for (int64_t p = pos_begin; p < pos_end; ++p) {
    float* row = out_host + (p - pos_begin) * static_cast<int64_t>(hd);
    const float position = static_cast<float>(p);
    for (int j = 0; j < half; ++j) {
      const float angle = position / den[j];
      row[2 * j] = cosf(angle);
      row[2 * j + 1] = sinf(angle);
    }
  }
  delete[] heap;
  return MLB_OK;
}
