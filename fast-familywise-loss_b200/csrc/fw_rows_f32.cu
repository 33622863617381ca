// Instances of run_rows (fw_rows.cuh): fp32 logits, gradient output.
#include "fw_rows.cuh"

namespace fwb200 {
template int run_rows<float, kOutGrad>(const RowArgs&, cudaStream_t, bool);
}  // namespace fwb200
