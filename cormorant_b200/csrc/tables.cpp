// Host builders of the unit tables.  Compiled with -ffp-contract=off so every
// double operation rounds on its own, as the reference's Python computes them.
#include <cmath>
#include <cstdint>
#include <cstring>

namespace corm {

// The activation of x in double: vectorop_act.py:60-73 (VectorOP.cpp act_fn),
// with the C library's exp / erf / tanh as the reference uses (host_nodes.py:156).
static double act_real(int act, double x, uint32_t alpha) {
  switch (act) {
    case 3: return x >= 0.0 ? x : x * ((double)(alpha & 0xFFFFu) / 65536.0);
    case 4: return x / (1.0 + std::exp(-x));
    case 5: return x * (0.5 * (1.0 + std::erf(x / std::sqrt(2.0))));
    case 6: {
      const double c = std::sqrt(2.0 / 3.141592653589793);
      const double cube = (x * x) * x;
      return x * (0.5 * (1.0 + std::tanh(c * (x + 0.044715 * cube))));
    }
    default: return x;
  }
}

// dtype.host_quantize at Q8.8 (dtype.py:214-219, 367-369): NaN -> 0, clip to
// [-128, 127.99609375], round half to even at 2^-8.
static int16_t host_quantize_q88(double v) {
  if (v != v) v = 0.0;
  if (v < -128.0) v = -128.0;
  if (v > 127.99609375) v = 127.99609375;
  return (int16_t)std::nearbyint(v * 256.0);
}

// vectorop_act.kernel_table (vectorop_act.py:92-95): out[raw + 32768].
void build_act_table(int act, uint32_t alpha, int16_t* out) {
  for (int r = -32768; r < 32768; r++) {
    const double x = (double)r / 256.0;
    out[r + 32768] = (act >= 3 && act <= 6) ? host_quantize_q88(act_real(act, x, alpha)) : (int16_t)r;
  }
}

// vectorop_smx.TAB (vectorop_smx.py:29): round(2^16 * 2^(-k / 4096)).
void build_smx_tab(int32_t* out) {
  for (int k = 0; k < 4096; k++) out[k] = (int32_t)std::nearbyint(65536.0 * std::pow(2.0, -(double)k / 4096.0));
}

// rowops_spec.table_image (rowops_spec.py:603-616): 4096 sigmoid words
// {(T[i+1] - T[i]) << 25 | T[i]} with T[i] = round(2^24 / (1 + exp(-i/256)))
// (rowops_spec.py:337-342), then 8192 rsqrt entries round(2^47 / sqrt((i +
// 0.5) 2^19)) for i >= 2048 (rowops_spec.py:91-101).
void build_rowops_image(uint8_t* out) {
  static int64_t T[4097];
  for (int i = 0; i <= 4096; i++) T[i] = (int64_t)std::nearbyint(16777216.0 / (1.0 + std::exp(-(double)i / 256.0)));
  std::memset(out, 0, 65536);
  for (int i = 0; i < 4096; i++) {
    const uint64_t d = (uint64_t)(T[i + 1] - T[i]) & 0xFFFFFFull, t = (uint64_t)T[i] & 0x1FFFFFFull;
    const uint64_t w = (d << 25) | t;
    std::memcpy(out + 8 * i, &w, 8);
  }
  for (int i = 2048; i < 8192; i++) {
    double y = std::nearbyint(std::ldexp(1.0, 47) / std::sqrt((i + 0.5) * 524288.0));
    if (y > 4294967295.0) y = 4294967295.0;
    const uint32_t v = (uint32_t)y;
    std::memcpy(out + 32768 + 4 * i, &v, 4);
  }
}

}  // namespace corm
