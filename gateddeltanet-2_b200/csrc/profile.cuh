// Launch-site hooks of the opt-in kernel timing (profile.cu).
#pragma once
#include <cuda_runtime.h>

namespace gdn2 {
enum KernelId { kKIntra = 0, kKScanFwd, kKScanBwd, kKBwdIntra, kKRecurrent, kKCp, kKScanFwdTc, kKScanBwdTc,
                kKLayerPrepFwd, kKLayerPrepBwd, kKNormGateFwd, kKNormGateBwd, kKSegFold, kKBwdFp32, kKFp32Aux, kNumKernels };
bool prof_on();
void prof_begin(int id, cudaStream_t s);
void prof_end(int id, cudaStream_t s);
struct ProfScope {
  int id;
  cudaStream_t s;
  ProfScope(int i, cudaStream_t st) : id(i), s(st) { prof_begin(id, s); }
  ~ProfScope() { prof_end(id, s); }
};
}  // namespace gdn2
