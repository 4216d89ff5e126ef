// placeholder; replaced by the tcgen05 GEMM
#include "common.cuh"
namespace ferrite { FERRITE_DEFINE_STATUS_READER(status_gemm) }
extern "C" int ferrite_gemm(void*, const void*, const void*, void*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int, int, int, int) { return ferrite::fail(FERRITE_UNSUPPORTED_DTYPE, "gemm: not built yet"); }
