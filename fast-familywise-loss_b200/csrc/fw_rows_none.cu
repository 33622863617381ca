// Instances of run_rows (fw_rows.cuh): forward only (no per-element output)
// for fp32, bf16 and fp16 logits.
#include "fw_rows.cuh"

namespace fwb200 {
template int run_rows<float, kOutNone>(const RowArgs&, cudaStream_t, bool);
template int run_rows<__nv_bfloat16, kOutNone>(const RowArgs&, cudaStream_t, bool);
template int run_rows<__half, kOutNone>(const RowArgs&, cudaStream_t, bool);
}  // namespace fwb200
