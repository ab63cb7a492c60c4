// Test harness: the device decoder of GGUF weight formats
// (gollama_b200/csrc/quant_formats.cuh) compiled as plain C++ for the host,
// so the tests compare the exact indexing and float32 arithmetic the kernel
// runs with the oracle, bit for bit, without a GPU.  Built by
// tests/test_quant.py with -ffp-contract=off; never linked into the library.
#include <cstddef>
#include <cstdint>

#include "../../gollama_b200/csrc/quant_formats.cuh"

extern "C" int qf_dequantize_host(const uint8_t* src, int type, float* dst, int64_t n) {
  const int be = glc::qf::block_elems(type);
  if (be == 0 || n % be || n % 4) return -1;
  for (int64_t g = 0; g < n / 4; ++g) glc::qf::dequant4(src, type, static_cast<size_t>(g), dst + 4 * g);
  return 0;
}
