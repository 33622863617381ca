// Instances of run_rows (fw_rows.cuh): fp32 logits, mask / candidate / class-shard outputs.
#include "fw_rows.cuh"

namespace fwb200 {
template int run_rows<float, kOutMask>(const RowArgs&, cudaStream_t, bool);
template int run_rows<float, kOutCand>(const RowArgs&, cudaStream_t, bool);
template int run_rows<float, kOutShard>(const RowArgs&, cudaStream_t, bool);
}  // namespace fwb200
