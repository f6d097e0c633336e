// The persistent decode-step kernel (decode_kernel.cuh) for layer matrices
// of one block type: Q4_0.
#include "decode_kernel.cuh"

namespace b200dec {
B200_DECODE_INSTANTIATE(PAI_B200_Q4_0)
}  // namespace b200dec
