// flashb: library-level C ABI (error reporting, device error word, launch helper).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "fb_common.cuh"

// The device error word: kernels whose bounded wait expires record an FB_ERR_* code here (first one wins).
__device__ unsigned g_fb_error_word;

namespace {
thread_local char t_msg[1024] = "";
std::mutex g_mu;
unsigned* g_err_ptr[64] = {nullptr};
int g_sms[64] = {0};
int g_pdl = -1;
thread_local int t_sm_budget = 0;   // SMs the calling thread's launches may size their grids for (0: all)
}  // namespace

namespace fbh {

void set_msg(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
}

unsigned* device_err_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fb_error_word) == cudaSuccess) g_err_ptr[dev] = (unsigned*)p;
  }
  return g_err_ptr[dev];
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!g_sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = n > 0 ? n : 148;
  }
  return g_sms[dev];
}

int tmap_rows(CUtensorMap* out, const void* base, long long rows, int K, int kc) {
  if (kc < 64 || kc % 64) {
    set_msg("tensor map: stage columns %d not a multiple of 64", kc);
    return FB_ERR_ARG;
  }
  return tmap_box(out, base, rows, K, 64, 8, kc / 64, true);
}

int tmap_box(CUtensorMap* out, const void* base, long long rows, int K, int inner, int box_rows, int box_blocks,
             bool swizzle128, long long ld) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  static std::map<std::tuple<uintptr_t, long long, int, int, int, int, int, long long>, CUtensorMap> cache;
  static std::mutex mu;
  if (ld == 0) ld = K;
  if (!base || rows < 1 || rows > (1ll << 31) || inner < 8 || inner % 8 || K < inner || K % inner || ld < K ||
      ld % 8 || box_rows < 1 || box_rows > 256 || box_blocks < 1 || box_blocks > 256 || (swizzle128 && inner != 64) ||
      (reinterpret_cast<uintptr_t>(base) & 15)) {
    set_msg("tensor map: bad matrix (rows %lld, K %d, ld %lld, block %d, box %d x %d, base %p)", rows, K, ld, inner,
            box_rows, box_blocks, base);
    return FB_ERR_ARG;
  }
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(reinterpret_cast<uintptr_t>(base), rows, K, inner, box_rows, box_blocks,
                                   swizzle128 ? 1 : 0, ld);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FB_OK;
  }
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn) {
      set_msg("tensor map: cuTensorMapEncodeTiled unavailable");
      return FB_ERR_CUDA;
    }
    enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)(K / inner)};
  const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)inner * 2};   // bytes: next row, next block
  const cuuint32_t box[3] = {(cuuint32_t)inner, (cuuint32_t)box_rows, (cuuint32_t)box_blocks};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_msg("tensor map: cuTensorMapEncodeTiled failed (%d) for rows %lld, K %d, box %d x %d x %d", (int)r, rows, K,
            inner, box_rows, box_blocks);
    return FB_ERR_CUDA;
  }
  cache.emplace(key, m);
  *out = m;
  return FB_OK;
}

int tmap_ln12(CUtensorMap* out, const void* data, long long N, int K, int box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  static std::map<std::tuple<uintptr_t, long long, int, int>, CUtensorMap> cache;
  static std::mutex mu;
  if (!data || N < 1 || N > (1ll << 31) || K < 1024 || K % 1024 || box_rows < 1 || box_rows > 256 ||
      (reinterpret_cast<uintptr_t>(data) & 15)) {
    set_msg("LN12 tensor map: bad matrix (N %lld, K %d, box rows %d, data %p)", N, K, box_rows, data);
    return FB_ERR_ARG;
  }
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(reinterpret_cast<uintptr_t>(data), N, K, box_rows);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FB_OK;
  }
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn) {
      set_msg("tensor map: cuTensorMapEncodeTiled unavailable");
      return FB_ERR_CUDA;
    }
    enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t G = (cuuint64_t)(K / 1024);
  const cuuint64_t dims[4] = {512, 3, G, (cuuint64_t)N};
  const cuuint64_t strides[3] = {512, 1536, 1536 * G};                  // bytes: next slot, next group, next row
  const cuuint32_t box[4] = {128, 3, 1, (cuuint32_t)box_rows};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(data), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_msg("LN12 tensor map: cuTensorMapEncodeTiled failed (%d) for N %lld, K %d", (int)r, N, K);
    return FB_ERR_CUDA;
  }
  cache.emplace(key, m);
  *out = m;
  return FB_OK;
}

int tmap_heads(CUtensorMap* out, const void* base, int B, int NH, long long S, long long sl, long long sh,
               long long sb) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  static std::map<std::tuple<uintptr_t, int, int, long long, long long, long long, long long>, CUtensorMap> cache;
  static std::mutex mu;
  if (!base || B < 1 || NH < 1 || S < 1 || S > (1ll << 31) || sl < 128 || (sl & 7) || (NH > 1 && (sh < 1 || (sh & 7))) ||
      (B > 1 && (sb < 1 || (sb & 7))) || (reinterpret_cast<uintptr_t>(base) & 15)) {
    set_msg("tensor map: bad head-major cache (B %d, heads %d, S %lld, strides %lld %lld %lld, base %p)", B, NH, S, sl,
            sh, sb, base);
    return FB_ERR_ARG;
  }
  // a dimension of extent 1 takes any valid stride
  if (NH == 1) sh = sl * S;
  if (B == 1) sb = sh * NH;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(reinterpret_cast<uintptr_t>(base), B, NH, S, sl, sh, sb);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FB_OK;
  }
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn) {
      set_msg("tensor map: cuTensorMapEncodeTiled unavailable");
      return FB_ERR_CUDA;
    }
    enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[5] = {8, (cuuint64_t)S, 16, (cuuint64_t)NH, (cuuint64_t)B};
  const cuuint64_t strides[4] = {(cuuint64_t)sl * 2, 16, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[5] = {8, 128, 16, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_msg("tensor map: cuTensorMapEncodeTiled failed (%d) for a head-major cache (B %d, heads %d, S %lld)", (int)r,
            B, NH, S);
    return FB_ERR_CUDA;
  }
  cache.emplace(key, m);
  *out = m;
  return FB_OK;
}

int grid_sms() {
  const int n = num_sms();
  return (t_sm_budget > 0 && t_sm_budget < n) ? t_sm_budget : n;
}

bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* e = getenv("FLASHB_PDL");
    g_pdl = (e && e[0] == '0') ? 0 : 1;
  }
  return g_pdl == 1;
}

int launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args, bool pdl,
               int cluster_x) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (pdl && pdl_enabled()) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 0) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = cluster_x;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = na ? at : nullptr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelExC(&cfg, func, args);
  if (e != cudaSuccess) {
    set_msg("kernel launch (grid %u x %u x %u, block %u, smem %zu): %s", grid.x, grid.y, grid.z, block.x, smem,
            cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

}  // namespace fbh

extern "C" const char* flashb_last_error(void) { return t_msg; }

extern "C" const char* flashb_version(void) { return "flashb 0.1 sm_100a"; }

extern "C" void flashb_set_pdl(int enable) { g_pdl = enable ? 1 : 0; }

extern "C" void flashb_set_sm_budget(int sms) { t_sm_budget = sms > 0 ? sms : 0; }

extern "C" int flashb_sm_budget(void) { return fbh::grid_sms(); }

extern "C" int flashb_device_error(int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fbh::set_msg("device error check: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, g_fb_error_word, sizeof(v));
  if (e != cudaSuccess) {
    fbh::set_msg("device error check: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_fb_error_word, &z, sizeof(z));
  }
  if (v) fbh::set_msg("device error word = %u (a bounded device-side wait expired)", v);
  return (int)v;
}
