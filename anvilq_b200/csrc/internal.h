// internal.h -- launchers shared between the translation units of libanvilq.so
// (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace anvilq {

// Batch-1 W4A16 GEMV on the TMA + cluster kernel (gemv_tma.cu).
bool gemv_tma_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                        int K, int N, int G);
size_t gemv_tma_workspace_bytes(int K, int N);
int launch_gemv_tma(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                    const uint16_t* bias, uint16_t* y, int K, int N, int G, void* workspace,
                    size_t workspace_bytes, int* dev_err, cudaStream_t stream, bool overlap_prior);

}  // namespace anvilq
