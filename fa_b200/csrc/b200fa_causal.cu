// b200fa_causal.cu -- the causal-mask kernels (B200FA_FLAG_CAUSAL): the
// kernel source of fa_kernel.cuh compiled with B200FA_CAUSAL = 1.  Query row
// i attends keys 0..i (top-left aligned, torch's is_causal); each work item
// stops at the diagonal key block of its last query block and the block
// crossing a row's diagonal is masked per row.  Launched by b200fa.cu.
#define B200FA_CAUSAL 1
// The roles that are plain (non-template) device functions get their own
// names here: the product translation unit defines the non-causal ones.
#define s_issuer_role s_issuer_role_causal
#define pv_issuer_role pv_issuer_role_causal
#define watch_role watch_role_causal
#define forward_role forward_role_causal
#define load_role load_role_causal
#include "fa_kernel.cuh"

using namespace b200fa;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    b200_fa_fp16_causal_kernel(const __grid_constant__ FwdParams p) {
  attention_fwd_body<0, false>(p);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    b200_fa_fp32_causal_kernel(const __grid_constant__ FwdParams p) {
  attention_fwd_body<1, false>(p);
}
