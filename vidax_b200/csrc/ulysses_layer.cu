// The DeepSpeed-Ulysses layer of vidax (sequence_parallel_self_attention,
// src/vidax/core/attention.py:341-388) behind the C ABI: head-slab packing,
// the NCCL exchanges and the attention kernel, pipelined by head slices over
// two streams, built on the library's own entry points (vx_ulysses_pack,
// vx_attn_fwd, vx_ulysses_unpack).
//
// NCCL is resolved at run time: the communicator a caller lends (torch's,
// for one) must be driven by the NCCL library that created it, so the one
// already loaded in the process is used (dlopen RTLD_NOLOAD), else
// libnccl.so.2 is loaded.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "vidax_cuda.h"
#include "vx_internal.h"

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_count)(const ncclComm_t, int*);
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int*);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  const char* (*error_string)(ncclResult_t);
};

const NcclApi* nccl_api(std::string* why) {
  static NcclApi api;
  static bool ok = false;
  static std::string err;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) {
      err = std::string("libnccl.so.2 not loadable: ") + dlerror();
      return;
    }
    bool all = true;
    auto sym = [&](const char* name) {
      void* f = dlsym(h, name);
      if (f == nullptr) {
        err = std::string("NCCL lacks ") + name;
        all = false;
      }
      return f;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
    api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(sym("ncclCommUserRank"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
    api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    ok = all;
  });
  if (!ok) {
    if (why) *why = err;
    return nullptr;
  }
  return &api;
}

int fail_msg(int code, const std::string& msg) { return vx_internal_fail(code, msg.c_str()); }

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", what, api->error_string(r));
  return vx_internal_fail(VX_ENCCL, buf);
}

int cuda_err(cudaError_t e, const char* what) {
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  return vx_internal_fail(VX_ECUDA, buf);
}

// Head counts of the pipelined slices of a rank's hg heads: a small first
// slice (its exchange is the one not hidden behind the kernel), then up to
// two larger ones (the same rule as the torch mirror's slices).
std::vector<int> head_slices(int hg) {
  if (hg <= 1) return {hg};
  const int first = std::max(1, hg / 5);
  const int rest = hg - first;
  if (rest <= 1) return {first, rest};
  return {first, rest - rest / 2, rest / 2};
}

constexpr int kEvents = 16;

}  // namespace

struct vx_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  bool owned = false;
  cudaStream_t side = nullptr;   // NCCL stream
  cudaEvent_t ev[kEvents] = {};
};

namespace {

int comm_setup(vx_comm* c, const NcclApi* api) {
  ncclResult_t r = api->comm_count(c->comm, &c->world);
  if (r != ncclSuccess) return nccl_fail(api, r, "ncclCommCount");
  r = api->comm_user_rank(c->comm, &c->rank);
  if (r != ncclSuccess) return nccl_fail(api, r, "ncclCommUserRank");
  cudaError_t e = cudaGetDevice(&c->device);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_err(e, "cudaStreamCreate");
  for (int i = 0; i < kEvents; ++i) {
    e = cudaEventCreateWithFlags(&c->ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_err(e, "cudaEventCreate");
  }
  return VX_OK;
}

// Equal-split all-to-all of up to three tensors in one NCCL group: chunk g
// (`chunk` elements) of send[t] goes to rank g, chunk g of recv[t] comes
// from rank g.
int exchange(const NcclApi* api, vx_comm* c, int n, void* const* send, void* const* recv,
             size_t chunk) {
  ncclResult_t r = api->group_start();
  if (r != ncclSuccess) return nccl_fail(api, r, "ncclGroupStart");
  for (int t = 0; t < n; ++t)
    for (int g = 0; g < c->world; ++g) {
      const size_t off = static_cast<size_t>(g) * chunk * 2;
      r = api->send(static_cast<const char*>(send[t]) + off, chunk, ncclBfloat16, g, c->comm,
                    c->side);
      if (r == ncclSuccess)
        r = api->recv(static_cast<char*>(recv[t]) + off, chunk, ncclBfloat16, g, c->comm, c->side);
      if (r != ncclSuccess) {
        api->group_end();
        return nccl_fail(api, r, "ncclSend / ncclRecv");
      }
    }
  r = api->group_end();
  if (r != ncclSuccess) return nccl_fail(api, r, "ncclGroupEnd");
  return VX_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Built-in workspace of vx_ulysses_attn_fwd_static, for callers that may not
// allocate device memory. One instance per GPU on which this library's
// device code is loaded, held until the process exits; every call on that
// GPU shares it.
constexpr int64_t kStaticWorkspaceBytes = 32ll << 20;
static __device__ __align__(256) unsigned char g_ulysses_static_ws[kStaticWorkspaceBytes];

namespace {

// Device address of g_ulysses_static_ws on the current device `dev`, looked
// up once per device. In host code the array's name is a host-side shadow,
// not a device address, so it is never handed to a kernel directly.
int static_workspace(int dev, void** out) {
  static std::mutex mu;
  static std::vector<void*> addr;
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0) return fail_msg(VX_EINVAL, "bad device");
  if (static_cast<size_t>(dev) >= addr.size()) addr.resize(dev + 1, nullptr);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ulysses_static_ws);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress(built-in Ulysses workspace)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return VX_OK;
}

}  // namespace

extern "C" {

int vx_comm_get_unique_id(char uid_out[128]) {
  std::string why;
  const NcclApi* api = nccl_api(&why);
  if (api == nullptr) return fail_msg(VX_ENCCL, why);
  if (uid_out == nullptr) return fail_msg(VX_EINVAL, "uid_out is NULL");
  ncclUniqueId id;
  ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(api, r, "ncclGetUniqueId");
  static_assert(sizeof(id.internal) == 128, "NCCL unique id is 128 bytes");
  memcpy(uid_out, id.internal, 128);
  return VX_OK;
}

int vx_comm_init(int32_t rank, int32_t world, const char uid[128], vx_comm** comm_out) {
  if (comm_out == nullptr || uid == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  if (world < 1 || rank < 0 || rank >= world) return fail_msg(VX_EINVAL, "rank must lie in [0, world)");
  std::string why;
  const NcclApi* api = nccl_api(&why);
  if (api == nullptr) return fail_msg(VX_ENCCL, why);
  ncclUniqueId id;
  memcpy(id.internal, uid, 128);
  vx_comm* c = new vx_comm();
  ncclResult_t r = api->comm_init_rank(&c->comm, world, id, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail(api, r, "ncclCommInitRank");
  }
  c->owned = true;
  int rc = comm_setup(c, api);
  if (rc != VX_OK) {
    vx_comm_destroy(c);
    return rc;
  }
  *comm_out = c;
  return VX_OK;
}

int vx_comm_wrap(void* nccl_comm, vx_comm** comm_out) {
  if (comm_out == nullptr || nccl_comm == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  std::string why;
  const NcclApi* api = nccl_api(&why);
  if (api == nullptr) return fail_msg(VX_ENCCL, why);
  vx_comm* c = new vx_comm();
  c->comm = static_cast<ncclComm_t>(nccl_comm);
  int rc = comm_setup(c, api);
  if (rc != VX_OK) {
    vx_comm_destroy(c);
    return rc;
  }
  *comm_out = c;
  return VX_OK;
}

int vx_comm_destroy(vx_comm* c) {
  if (c == nullptr) return VX_OK;
  int rc = VX_OK;
  if (c->side != nullptr) {
    cudaStreamSynchronize(c->side);
    cudaStreamDestroy(c->side);
  }
  for (int i = 0; i < kEvents; ++i)
    if (c->ev[i] != nullptr) cudaEventDestroy(c->ev[i]);
  if (c->owned && c->comm != nullptr) {
    const NcclApi* api = nccl_api(nullptr);
    if (api != nullptr) {
      ncclResult_t r = api->comm_destroy(c->comm);
      if (r != ncclSuccess) rc = nccl_fail(api, r, "ncclCommDestroy");
    }
  }
  delete c;
  return rc;
}

int vx_ulysses_workspace_size(const vx_ulysses_args* a, int32_t world, int64_t* bytes_out) {
  if (a == nullptr || bytes_out == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  if (world < 1 || a->seq_local < 0 || a->heads <= 0 || a->head_dim <= 0)
    return fail_msg(VX_EINVAL, "bad sizes");
  const long long hg = (a->heads + world - 1) / world;
  const long long slab = static_cast<long long>(world) * a->seq_local * hg * a->head_dim * 2;
  // q, k, v send and receive slabs, the attention output and its received
  // copy; one int for the key count, padded to 256 bytes in front
  *bytes_out = 256 + 8 * ((slab + 255) / 256 * 256);
  return VX_OK;
}

int vx_ulysses_attn_fwd(const vx_ulysses_args* a, vx_comm* c, vx_stream_t stream) {
  if (a == nullptr || c == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  std::string why;
  const NcclApi* api = nccl_api(&why);
  if (api == nullptr) return fail_msg(VX_ENCCL, why);
  const int P = c->world;
  if (a->batch < 0 || a->seq_local < 0 || a->heads <= 0 || a->heads > 65535)
    return fail_msg(VX_EINVAL, "bad sizes");
  if (a->head_dim != 64 && a->head_dim != 128)
    return fail_msg(VX_EUNSUPPORTED, "head_dim must be 64 or 128");
  if (a->batch == 0 || a->seq_local == 0) return VX_OK;
  const long long S = static_cast<long long>(P) * a->seq_local;
  if (S > 0x7fffffffLL) return fail_msg(VX_EUNSUPPORTED, "sequence too long");
  if (a->valid_len < 0 || a->valid_len > S) return fail_msg(VX_EINVAL, "valid_len outside [0, world * seq_local]");
  int64_t need = 0;
  int rc = vx_ulysses_workspace_size(a, P, &need);
  if (rc != VX_OK) return rc;
  if (a->workspace == nullptr || a->workspace_bytes < need)
    return fail_msg(VX_EINVAL, "workspace missing or smaller than vx_ulysses_workspace_size");
  if (reinterpret_cast<uintptr_t>(a->workspace) % 256 != 0)
    return fail_msg(VX_EINVAL, "workspace must be 256-byte aligned");
  const void* ptrs[4] = {a->q, a->k, a->v, a->o};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return fail_msg(VX_EINVAL, "q, k, v, o must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  if (dev != c->device) return fail_msg(VX_EINVAL, "the communicator belongs to another device");

  const int H = a->heads, D = a->head_dim, S_loc = a->seq_local;
  const int Hg = (H + P - 1) / P;
  const std::vector<int> sizes = head_slices(Hg);
  const int n = static_cast<int>(sizes.size());
  std::vector<int> offs(n, 0);
  for (int j = 1; j < n; ++j) offs[j] = offs[j - 1] + sizes[j - 1];
  const size_t slab_elems = static_cast<size_t>(P) * S_loc * Hg * D;
  const size_t slab_bytes = (slab_elems * 2 + 255) / 256 * 256;
  char* ws = static_cast<char*>(a->workspace);
  int* kv_len = reinterpret_cast<int*>(ws);
  char* send[3] = {ws + 256, ws + 256 + slab_bytes, ws + 256 + 2 * slab_bytes};
  char* recv[3] = {ws + 256 + 3 * slab_bytes, ws + 256 + 4 * slab_bytes, ws + 256 + 5 * slab_bytes};
  char* o_send = ws + 256 + 6 * slab_bytes;
  char* o_recv = ws + 256 + 7 * slab_bytes;
  // slice j of a slab: (P, S_loc, sizes[j], D) at element offset P * S_loc * offs[j] * D
  auto slice_ptr = [&](char* base, int j) {
    return base + static_cast<size_t>(P) * S_loc * offs[j] * D * 2;
  };
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool masked = a->valid_len > 0 && a->valid_len < S;
  if (masked) {
    const int kv = a->valid_len;
    e = cudaMemcpyAsync(kv_len, &kv, sizeof(int), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_err(e, "cudaMemcpyAsync(valid_len)");
  }
  cudaEvent_t* ev = c->ev;  // [0]: packed, [1 + j]: slice j received, [5 + j]: attention j, [9 + j]: slice j sent back
  for (int b = 0; b < a->batch; ++b) {
    // 1. per slice, pack this rank's tokens' heads of every rank group
    for (int j = 0; j < n; ++j) {
      vx_head_slab_args pk;
      memset(&pk, 0, sizeof(pk));
      pk.num_tensors = 3;
      const void* src[3] = {a->q, a->k, a->v};
      const int64_t* strd[3] = {a->q_stride, a->k_stride, a->v_stride};
      for (int t = 0; t < 3; ++t) {
        pk.src[t] = static_cast<const char*>(src[t]) + b * strd[t][0] * 2;
        pk.dst[t] = slice_ptr(send[t], j);
        pk.stride[t][0] = strd[t][1];
        pk.stride[t][1] = strd[t][2];
      }
      pk.seq = S_loc;
      pk.heads = H;
      pk.head_dim = D;
      pk.groups = P;
      pk.slab_heads = sizes[j];
      pk.group_stride = Hg;
      pk.head_offset = offs[j];
      pk.group_valid = sizes[j];
      if ((rc = vx_ulysses_pack(&pk, stream)) != VX_OK) return rc;
    }
    if ((e = cudaEventRecord(ev[0], st)) != cudaSuccess) return cuda_err(e, "cudaEventRecord");
    if ((e = cudaStreamWaitEvent(c->side, ev[0], 0)) != cudaSuccess) return cuda_err(e, "cudaStreamWaitEvent");
    // 2. tokens -> heads exchange of slice j on the NCCL stream, one slice ahead
    auto start_in = [&](int j) -> int {
      void* s3[3] = {slice_ptr(send[0], j), slice_ptr(send[1], j), slice_ptr(send[2], j)};
      void* r3[3] = {slice_ptr(recv[0], j), slice_ptr(recv[1], j), slice_ptr(recv[2], j)};
      int r = exchange(api, c, 3, s3, r3, static_cast<size_t>(S_loc) * sizes[j] * D);
      if (r != VX_OK) return r;
      cudaError_t e2 = cudaEventRecord(ev[1 + j], c->side);
      return e2 == cudaSuccess ? VX_OK : cuda_err(e2, "cudaEventRecord");
    };
    if ((rc = start_in(0)) != VX_OK) return rc;
    for (int j = 0; j < n; ++j) {
      if (j + 1 < n && (rc = start_in(j + 1)) != VX_OK) return rc;
      // 3. attention over the full sequence for slice j's heads; (1, S, hs, D)
      //    in and out, the output already the heads -> tokens send layout
      if ((e = cudaStreamWaitEvent(st, ev[1 + j], 0)) != cudaSuccess) return cuda_err(e, "cudaStreamWaitEvent");
      const int hs = sizes[j];
      vx_attn_args at;
      memset(&at, 0, sizeof(at));
      at.q = slice_ptr(recv[0], j);
      at.k = slice_ptr(recv[1], j);
      at.v = slice_ptr(recv[2], j);
      at.o = slice_ptr(o_send, j);
      const int64_t str[3] = {S * hs * D, static_cast<int64_t>(hs) * D, D};
      for (int i = 0; i < 3; ++i) at.q_stride[i] = at.k_stride[i] = at.v_stride[i] = at.o_stride[i] = str[i];
      at.batch = 1;
      at.seq_q = at.seq_k = static_cast<int32_t>(S);
      at.heads_q = at.heads_kv = hs;
      at.head_dim = D;
      at.scale = a->scale;
      at.kv_len = masked ? kv_len : nullptr;
      at.schedule = VX_SCHED_DYNAMIC;  // NCCL's kernels hold SMs meanwhile
      if ((rc = vx_attn_fwd(&at, stream)) != VX_OK) return rc;
      if ((e = cudaEventRecord(ev[5 + j], st)) != cudaSuccess) return cuda_err(e, "cudaEventRecord");
      // 4. heads -> tokens exchange of slice j behind it on the NCCL stream
      if ((e = cudaStreamWaitEvent(c->side, ev[5 + j], 0)) != cudaSuccess) return cuda_err(e, "cudaStreamWaitEvent");
      void* so[1] = {slice_ptr(o_send, j)};
      void* ro[1] = {slice_ptr(o_recv, j)};
      if ((rc = exchange(api, c, 1, so, ro, static_cast<size_t>(S_loc) * hs * D)) != VX_OK) return rc;
      if ((e = cudaEventRecord(ev[9 + j], c->side)) != cudaSuccess) return cuda_err(e, "cudaEventRecord");
    }
    // 5. unpack every slice into this rank's (S_loc, H, D) output rows
    if ((e = cudaStreamWaitEvent(st, ev[9 + n - 1], 0)) != cudaSuccess) return cuda_err(e, "cudaStreamWaitEvent");
    for (int j = 0; j < n; ++j) {
      vx_head_slab_args up;
      memset(&up, 0, sizeof(up));
      up.num_tensors = 1;
      up.src[0] = slice_ptr(o_recv, j);
      up.dst[0] = static_cast<char*>(a->o) + b * a->o_stride[0] * 2;
      up.stride[0][0] = a->o_stride[1];
      up.stride[0][1] = a->o_stride[2];
      up.seq = S_loc;
      up.heads = H;
      up.head_dim = D;
      up.groups = P;
      up.slab_heads = sizes[j];
      up.group_stride = Hg;
      up.head_offset = offs[j];
      up.group_valid = sizes[j];
      if ((rc = vx_ulysses_unpack(&up, stream)) != VX_OK) return rc;
    }
  }
  return VX_OK;
}

int vx_ulysses_attn_fwd_static(const vx_ulysses_args* a, vx_comm* c, vx_stream_t stream) {
  if (a == nullptr || c == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  int64_t need = 0;
  int rc = vx_ulysses_workspace_size(a, c->world, &need);
  if (rc != VX_OK) return rc;
  if (need > kStaticWorkspaceBytes) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "this call needs %lld bytes of workspace; the built-in workspace holds %lld "
             "(32 MiB): pass a workspace to vx_ulysses_attn_fwd instead",
             static_cast<long long>(need), static_cast<long long>(kStaticWorkspaceBytes));
    return fail_msg(VX_EINVAL, buf);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  if (dev != c->device) return fail_msg(VX_EINVAL, "the communicator belongs to another device");
  void* ws = nullptr;
  if ((rc = static_workspace(dev, &ws)) != VX_OK) return rc;
  // The layer writes every workspace byte it reads in the same call (the key
  // count, the zero-filled padding heads of the packed slabs), so nothing
  // needs clearing between calls.
  vx_ulysses_args b = *a;
  b.workspace = ws;
  b.workspace_bytes = kStaticWorkspaceBytes;
  return vx_ulysses_attn_fwd(&b, c, stream);
}

}  // extern "C"
