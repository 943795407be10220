// Persistent decode step instantiated for head_dim 128, f32 KV cache.
#include "decode_step_impl.cuh"

namespace sb {

int ds_limit_128_f32(int rep, int *limit) { return ds_limit_rep<128, float>(rep, limit); }
int ds_launch_128_f32(const DsArgs &a, int rep, cudaStream_t st) { return ds_rep<128, float>(a, rep, st); }

}  // namespace sb
