// placeholder; replaced by the tcgen05 attention kernels
#include "common.cuh"
namespace ferrite { FERRITE_DEFINE_STATUS_READER(status_attention) }
extern "C" {
int ferrite_attn_fwd(void*, const void*, const void*, const void*, void*, float*, int64_t, int64_t, int64_t, int64_t, int64_t, float, int, int, int, int) { return ferrite::fail(FERRITE_UNSUPPORTED_DTYPE, "attn: not built yet"); }
int ferrite_attn_bwd_prep(void*, const void*, const void*, float*, int64_t, int64_t, int64_t, int64_t, int) { return ferrite::fail(FERRITE_UNSUPPORTED_DTYPE, "attn: not built yet"); }
int ferrite_attn_bwd_dkv(void*, const void*, const void*, const void*, const void*, const float*, const float*, void*, void*, int64_t, int64_t, int64_t, int64_t, int64_t, float, int, int, int, int) { return ferrite::fail(FERRITE_UNSUPPORTED_DTYPE, "attn: not built yet"); }
int ferrite_attn_bwd_dq(void*, const void*, const void*, const void*, const void*, const float*, const float*, void*, int64_t, int64_t, int64_t, int64_t, int64_t, float, int, int, int, int) { return ferrite::fail(FERRITE_UNSUPPORTED_DTYPE, "attn: not built yet"); }
}
