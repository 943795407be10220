// Persistent decode step instantiated for head_dim 128, bf16 KV cache.
#include "decode_step_impl.cuh"

namespace sb {

int ds_limit_128_bf16(int rep, int *limit) { return ds_limit_rep<128, __nv_bfloat16>(rep, limit); }
int ds_launch_128_bf16(const DsArgs &a, int rep, cudaStream_t st) { return ds_rep<128, __nv_bfloat16>(a, rep, st); }

}  // namespace sb
