// Instances of run_rows (fw_rows.cuh): fp32 logits, gradient output with the support columns listed.
#include "fw_rows.cuh"

namespace fwb200 {
template int run_rows<float, kOutGradCols>(const RowArgs&, cudaStream_t, bool);
}  // namespace fwb200
