// libvidax_cuda.so: the C ABI declared in include/vidax_cuda.h.
//
// Host side of the sm_100a attention kernels: argument validation, TMA
// tensor-map construction over the caller's strided tensors, launch
// configuration and the per-device status word the kernels report bounded-
// wait timeouts into. Nothing here allocates device memory.
#include "vidax_cuda.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cmath>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "attn_sm100.cuh"

namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kMaxDevices = 64;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(VX_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

}  // namespace

// Device status word: kernels OR timeout codes into it (one instance per
// device context).
__device__ int g_vx_status;

namespace {

std::mutex g_mu;
int* g_status_ptr[kMaxDevices] = {};
std::set<std::pair<const void*, int>> g_attr_set;

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(VX_EUNSUPPORTED, "device id %d", *dev);
  return VX_OK;
}

int status_word(int dev, int** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_vx_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    g_status_ptr[dev] = static_cast<int*>(ptr);
  }
  *out = g_status_ptr[dev];
  return VX_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      cached = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (cached == nullptr) {
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    return fail(VX_ECUDA, "cuTensorMapEncodeTiled not available from the driver");
  }
  *fn = cached;
  return VX_OK;
}

// Tiled bf16 tensor map with 128B swizzle; dims[0] is contiguous. `strides`
// are the byte strides of dims 1..rank-1.
int make_tmap(CUtensorMap* tm, const void* base, int rank, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box) {
  EncodeTiledFn enc;
  int rc = get_encode_fn(&enc);
  if (rc != VX_OK) return rc;
  cuuint32_t elem_str[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                   const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                   reinterpret_cast<const cuuint64_t*>(strides),
                   reinterpret_cast<const cuuint32_t*>(box), elem_str,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VX_EINVAL, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return VX_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// BSHD operand -> 4-D map {D, H, S, B} with a {64, 1, 128, 1} box.
int bshd_tmap(CUtensorMap* tm, const char* name, const void* ptr, const int64_t* st, int B,
              int S, int H, int D) {
  if (ptr == nullptr) return fail(VX_EINVAL, "%s is NULL", name);
  if (!aligned16(ptr)) return fail(VX_EINVAL, "%s must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i) {
    if (st[i] <= 0 || (st[i] * 2) % 16 != 0)
      return fail(VX_EINVAL, "%s stride[%d]=%lld must be a positive multiple of 8 elements", name,
                  i, (long long)st[i]);
  }
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)S, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap(tm, ptr, 4, dims, strides, box);
}

int prepare_kernel(const void* fn, int dev, size_t smem) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_attr_set.count({fn, dev}) == 0) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
    g_attr_set.insert({fn, dev});
  }
  return VX_OK;
}

}  // namespace

extern "C" {

int vx_version(void) { return kVersion; }

const char* vx_last_error(void) { return g_last_error.c_str(); }

int vx_device_status(int* status_out, int clear) {
  int dev;
  int rc = current_device(&dev);
  if (rc != VX_OK) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_vx_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status)");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_vx_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status)");
  }
  if (status_out) *status_out = v;
  return VX_OK;
}

int vx_attn_fwd(const vx_attn_args* a, vx_stream_t stream) {
  using namespace vx::attn;
  if (a == nullptr) return fail(VX_EINVAL, "args is NULL");
  if (a->batch < 0 || a->seq_q < 0 || a->seq_k < 0 || a->heads_q <= 0 || a->heads_kv <= 0)
    return fail(VX_EINVAL, "negative or zero size (B=%d Sq=%d Sk=%d Hq=%d Hkv=%d)", a->batch,
                a->seq_q, a->seq_k, a->heads_q, a->heads_kv);
  if (a->heads_q % a->heads_kv != 0)
    return fail(VX_EINVAL, "heads_q (%d) must be a multiple of heads_kv (%d)", a->heads_q,
                a->heads_kv);
  if (a->head_dim != kHeadDim)
    return fail(VX_EUNSUPPORTED, "head_dim %d (this build implements %d)", a->head_dim, kHeadDim);
  if (!(a->scale > 0.f) || !std::isfinite(a->scale))
    return fail(VX_EUNSUPPORTED, "softmax scale must be finite and > 0 (got %g)", (double)a->scale);
  if (a->batch > 65535 || a->heads_q > 65535)
    return fail(VX_EUNSUPPORTED, "batch and heads must be <= 65535");
  if (a->batch == 0 || a->seq_q == 0) return VX_OK;
  if (a->o == nullptr) return fail(VX_EINVAL, "o is NULL");
  if (!aligned16(a->o)) return fail(VX_EINVAL, "o must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (a->o_stride[i] <= 0 || a->o_stride[i] % 8 != 0)
      return fail(VX_EINVAL, "o stride[%d]=%lld must be a positive multiple of 8 elements", i,
                  (long long)a->o_stride[i]);

  int dev;
  int rc = current_device(&dev);
  if (rc != VX_OK) return rc;
  int* status = nullptr;
  if ((rc = status_word(dev, &status)) != VX_OK) return rc;

  // Key tensors need at least one row for a valid tensor map; with seq_k == 0
  // every output row is zero and no K/V tile is loaded.
  CUtensorMap tq, tk, tv;
  if ((rc = bshd_tmap(&tq, "q", a->q, a->q_stride, a->batch, a->seq_q, a->heads_q, kHeadDim)) != VX_OK)
    return rc;
  if (a->seq_k > 0) {
    if ((rc = bshd_tmap(&tk, "k", a->k, a->k_stride, a->batch, a->seq_k, a->heads_kv, kHeadDim)) != VX_OK)
      return rc;
    if ((rc = bshd_tmap(&tv, "v", a->v, a->v_stride, a->batch, a->seq_k, a->heads_kv, kHeadDim)) != VX_OK)
      return rc;
  } else {
    tk = tq;  // never dereferenced: with no keys every output row is zero
    tv = tq;
  }

  DenseParams p;
  p.o = static_cast<__nv_bfloat16*>(a->o);
  p.o_sb = a->o_stride[0];
  p.o_ss = a->o_stride[1];
  p.o_sh = a->o_stride[2];
  p.lse = a->lse;
  p.kv_len = a->kv_len;
  p.status = status;
  p.B = a->batch;
  p.Sq = a->seq_q;
  p.Sk = a->seq_k;
  p.H = a->heads_q;
  p.Hkv = a->heads_kv;
  p.scale_log2 = a->scale * 1.4426950408889634f;

  auto kern = attn_fwd_kernel<DenseGeo>;
  if ((rc = prepare_kernel(reinterpret_cast<const void*>(kern), dev, kSmemBytes)) != VX_OK) return rc;
  dim3 grid((a->seq_q + 2 * kBlockM - 1) / (2 * kBlockM), a->heads_q, a->batch);
  kern<<<grid, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd launch");
  return VX_OK;
}

}  // extern "C"
