// Library plumbing behind the C ABI: thread-local last-error string, version,
// device status word, per-device SM count cache, host-side fault injection and
// TMA descriptor encoding (through the driver entry point, so the library needs
// no link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace ferrite {

namespace {
thread_local std::string t_last_error;
std::mutex g_mu;
int g_sm_count[64] = {0};
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int num_sms(int device) {
  if (device < 0 || device >= 64) return 148;
  int v = __atomic_load_n(&g_sm_count[device], __ATOMIC_ACQUIRE);
  if (v > 0) return v;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) !=
          cudaSuccess ||
      n <= 0)
    n = 148;
  __atomic_store_n(&g_sm_count[device], n, __ATOMIC_RELEASE);
  return n;
}

int injected_fault(const char* op) {
  const char* env = std::getenv("FERRITE_FAULT_INJECT");
  if (env == nullptr || *env == '\0') return 0;
  std::string list(env);
  if (list == "all")
    return fail(FERRITE_INJECTED_FAULT, "%s: injected fault (FERRITE_FAULT_INJECT=all)", op);
  size_t start = 0;
  while (start <= list.size()) {
    size_t end = list.find(',', start);
    if (end == std::string::npos) end = list.size();
    if (list.compare(start, end - start, op) == 0)
      return fail(FERRITE_INJECTED_FAULT, "%s: injected fault (FERRITE_FAULT_INJECT)", op);
    start = end + 1;
  }
  return 0;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(FERRITE_LAUNCH_FAILED, "%s: launch failed: %s", what,
                cudaGetErrorString(e));
  return FERRITE_OK;
}

cudaError_t launch_k(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     void** args) {
  static const bool pdl = [] {
    const char* e = std::getenv("FERRITE_PDL");
    return !(e && *e && std::atoi(e) == 0);
  }();
  if (!pdl) return cudaLaunchKernel(func, grid, block, args, smem, s);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, func, args);
}

cudaError_t launch_k_cluster(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             void** args, unsigned cluster_x) {
  static const bool pdl = [] {
    const char* e = std::getenv("FERRITE_PDL");
    return !(e && *e && std::atoi(e) == 0);
  }();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelExC(&cfg, func, args);
}

int max_active_clusters(const void* func, dim3 block, size_t smem, unsigned cluster_x) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster_x, 1, 1);
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, func, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

static int load_encoder() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_encode_tiled) return FERRITE_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                          cudaEnableDefault, &q);
  if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
    return fail(FERRITE_LAUNCH_FAILED,
                "cuTensorMapEncodeTiled unavailable from the driver");
  g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return FERRITE_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  if (int rc = load_encoder()) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA base %p is not 16-byte aligned", base);
  if (row_stride_bytes % 16 != 0)
    return fail(FERRITE_BAD_ALIGNMENT,
                "TMA row stride %llu bytes is not a multiple of 16",
                (unsigned long long)row_stride_bytes);
  if ((box_inner * (uint32_t)elem_bytes) % 16 != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA box inner extent not 16-byte multiple");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(map, dtype, 2, const_cast<void*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FERRITE_BAD_SHAPE,
                "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu "
                "box %u x %u",
                (int)r, (unsigned long long)inner, (unsigned long long)outer,
                (unsigned long long)row_stride_bytes, box_inner, box_outer);
  return FERRITE_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                 uint32_t box1, uint32_t box2, CUtensorMapSwizzle swizzle) {
  if (int rc = load_encoder()) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA base %p is not 16-byte aligned", base);
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA strides must be multiples of 16 bytes");
  if ((box0 * (uint32_t)elem_bytes) % 16 != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA box inner extent not 16-byte multiple");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode_tiled(map, dtype, 3, const_cast<void*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FERRITE_BAD_SHAPE, "cuTensorMapEncodeTiled (3d) failed (%d)", (int)r);
  return FERRITE_OK;
}

int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, const uint64_t dims[4], const uint64_t strides_bytes[3],
                 const uint32_t box[4], CUtensorMapSwizzle swizzle) {
  if (int rc = load_encoder()) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA base %p is not 16-byte aligned", base);
  for (int i = 0; i < 3; ++i)
    if (strides_bytes[i] % 16 != 0 || strides_bytes[i] == 0 || strides_bytes[i] >= (1ull << 40))
      return fail(FERRITE_BAD_ALIGNMENT, "TMA stride %d (%llu bytes) must be a positive multiple of 16 below 2^40",
                  i + 1, (unsigned long long)strides_bytes[i]);
  if ((box[0] * (uint32_t)elem_bytes) % 16 != 0)
    return fail(FERRITE_BAD_ALIGNMENT, "TMA box inner extent not 16-byte multiple");
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode_tiled(map, dtype, 4, const_cast<void*>(base), d, st, bx, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FERRITE_BAD_SHAPE, "cuTensorMapEncodeTiled (4d) failed (%d)", (int)r);
  return FERRITE_OK;
}

}  // namespace ferrite

extern "C" {

const char* ferrite_last_error(void) { return ferrite::t_last_error.c_str(); }

const char* ferrite_version(void) { return "ferrite_b200 0.1.0 sm_100a"; }

int ferrite_device_status(void* stream, int clear) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess)
    return ferrite::fail(FERRITE_LAUNCH_FAILED, "stream sync failed: %s",
                         cudaGetErrorString(e));
  int v = 0;
  for (int st : {ferrite::status_gemm(clear), ferrite::status_attention(clear),
                 ferrite::status_rmsnorm(clear)})
    if (v == 0 && st != 0) v = st;
  if (v != 0)
    return ferrite::fail(v, "device reported status %d (a bounded wait expired)", v);
  return FERRITE_OK;
}

}  // extern "C"
