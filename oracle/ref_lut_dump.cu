// Prints the reference's own FP8(E4M3)->fp16 table, built on the host by the
// reference's helpers (src/fp8imma/fp8imma_internal.cuh:49-70, the same calls
// init_fp8_e4m3_lut makes in src/fp8imma/fp8_lut.cu:16-18). Test
// infrastructure: its output is the committed golden file
// tests/golden/lut_e4m3_ref.txt. Runs on the CPU; touches no device.
#include "fp8imma_internal.cuh"

#include <cstdio>

int main() {
  for (int i = 0; i < 256; ++i) {
    uint16_t bits = fp8imma_internal::f32_to_f16_bits(fp8imma_internal::fp8_e4m3_to_f32((uint8_t)i));
    std::printf("%d %04x\n", i, (unsigned)bits);
  }
  return 0;
}
