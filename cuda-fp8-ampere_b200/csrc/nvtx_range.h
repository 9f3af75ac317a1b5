// NVTX ranges around the public entry points (built with -DFP8IMMA_NVTX, the
// default): each call shows up as a named range in Nsight timelines. NVTX is
// header-only; without a tool attached a range costs a few nanoseconds.
#pragma once

#ifdef FP8IMMA_NVTX
#include <nvtx3/nvToolsExt.h>

struct Fp8immaRange {
  explicit Fp8immaRange(const char* name) { nvtxRangePushA(name); }
  ~Fp8immaRange() { nvtxRangePop(); }
  Fp8immaRange(const Fp8immaRange&) = delete;
  Fp8immaRange& operator=(const Fp8immaRange&) = delete;
};
#define FP8IMMA_RANGE(name) Fp8immaRange fp8imma_nvtx_range_(name)
#else
#define FP8IMMA_RANGE(name) \
  do {                      \
  } while (0)
#endif
