// Split-KV decode kernel (placeholder until implemented): never eligible.
#pragma once
#include "rdna/forward.hpp"
#include <cuda_runtime.h>
namespace rdna {
namespace decode {
inline bool eligible(uint32_t, uint32_t, uint32_t) { return false; }
inline int launch_f16(char*, const ForwardParams&, cudaStream_t) { return -1; }
}  // namespace decode
}  // namespace rdna
