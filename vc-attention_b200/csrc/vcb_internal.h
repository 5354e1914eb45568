// Declarations shared by the translation units of libvcb.so.
#pragma once

#include "vcb_common.cuh"

namespace vcb {

// vcb_qk.cu
size_t qk_workspace_bytes(int64_t heads, int64_t sk);
int qk_run(const vcb_qk_args* p, bool quantise, cudaStream_t st);

// vcb_vprep.cu
int vprep_run(const vcb_v_args* p, cudaStream_t st);

// vcb_cluster.cu
size_t group_workspace_bytes(int64_t heads, int64_t s, int d, int clusters);
int group_run(const vcb_group_args* p, cudaStream_t st);

// vcb_api.cu: the SM count of the current device (cached)
int sm_count();

// vcb_attn.cu (ExpCast modes; dispatches the others to vcb_attn_exp.cu)
int attn_run(const vcb_attn_args* p, const vcb_attn_probe* probe, cudaStream_t st);
// vcb_attn_exp.cu (exp modes: fp8_control, v_smooth)
int attn_exp_run(const vcb_attn_args* p, const vcb_attn_probe* probe, cudaStream_t st);
int wait_selftest_run(int complete, const void* src, int32_t* status, int32_t* report, cudaStream_t st);

// vcb_expcast.cu
int expcast_run(const float* x, uint8_t* codes, int64_t n, cudaStream_t st);

}  // namespace vcb
