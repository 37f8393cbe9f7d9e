// k_gemm_tc.cu -- tcgen05 BF16 GEMM (placeholder until the kernel lands).
#include "kernels.h"

namespace s2b {

bool gemm_tc_supported(int, int, int, int, int) { return false; }
int gemm_tc(const void*, int, const void*, int, int, int, int, const GemmEpi&, cudaStream_t, int*) { return -1; }

int awa_init_device();
int kernels_init_device() { return awa_init_device(); }

}  // namespace s2b
