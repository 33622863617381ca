// Instances of run_rows (fw_rows.cuh): bf16 logits, gradient outputs.
#include "fw_rows.cuh"

namespace fwb200 {
template int run_rows<__nv_bfloat16, kOutGrad>(const RowArgs&, cudaStream_t, bool);
template int run_rows<__nv_bfloat16, kOutGradCols>(const RowArgs&, cudaStream_t, bool);
}  // namespace fwb200
