// Persistent decode step instantiated for head_dim 64, f32 KV cache.
#include "decode_step_impl.cuh"

namespace sb {

int ds_limit_64_f32(int rep, int *limit) { return ds_limit_rep<64, float>(rep, limit); }
int ds_launch_64_f32(const DsArgs &a, int rep, cudaStream_t st) { return ds_rep<64, float>(a, rep, st); }

}  // namespace sb
