// Instances of run_rows (fw_rows.cuh): fp16 logits, gradient outputs.
#include "fw_rows.cuh"

namespace fwb200 {
template int run_rows<__half, kOutGrad>(const RowArgs&, cudaStream_t, bool);
template int run_rows<__half, kOutGradCols>(const RowArgs&, cudaStream_t, bool);
}  // namespace fwb200
