/*
 * vidax_cuda.h -- C ABI of libvidax_cuda.so, the B200 (sm_100a) implementation
 * of vidax's attention hot path.
 *
 * Every compute entry point takes plain device pointers, sizes and element
 * strides and a CUDA stream; none allocates or frees device memory, none
 * synchronises the host. The exceptions are the communicator handles
 * (vx_comm_init / vx_comm_wrap create a host object, an internal stream and
 * events; vx_comm_destroy waits for that stream), vx_ipc_open / vx_ipc_close
 * (map / unmap another process's allocation) and the status / self-test
 * calls, which synchronise. Return value: VX_OK or a VX_E* code;
 * vx_last_error() gives the message of the last failure on the calling
 * thread.
 *
 * Layouts follow vidax: attention tensors are BSHD (batch, seq, heads,
 * head_dim) with head_dim contiguous; neighborhood tensors are
 * (B, T, H, W, heads, head_dim). Element type bf16 in and out, fp32 softmax.
 */
#ifndef VIDAX_CUDA_H_
#define VIDAX_CUDA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* vx_stream_t;

enum {
  VX_OK = 0,
  VX_EINVAL = 1,        /* bad argument: shape, stride, alignment, null pointer */
  VX_EUNSUPPORTED = 2,  /* valid request this build does not implement */
  VX_ECUDA = 3,         /* CUDA runtime / driver error */
  VX_ENCCL = 4,         /* NCCL error (vx_comm_*, vx_ulysses_attn_fwd) */
  VX_ETIMEOUT = 5,      /* a bounded device-side wait expired (see vx_device_status) */
};

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int vx_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* vx_last_error(void);

/*
 * Reads (and optionally clears) the device status word of the current CUDA
 * device: 0 when every kernel ran to completion, else an OR of
 * 1 (load wait timed out), 2 (MMA wait), 4 (softmax wait), 8 (drain),
 * 32 (a vx_peer_barrier wait).
 * Synchronises the device. Returns VX_OK or VX_ECUDA.
 */
int vx_device_status(int* status_out, int clear);

/* ----------------------------------------------------------------------
 * Full (non-causal) attention:  o = softmax(scale * q k^T) v   per (b, h).
 *
 * Replaces the kernel call behind vidax.core.attention.dot_product_attention
 * (src/vidax/core/attention.py:467-533), local_attention (:321-338) and the
 * per-device flash call inside _flash_attention_tpu (:212-288): the Pallas
 * flash_attention / splash_attention custom calls on TPU and
 * jax.nn.dot_product_attention elsewhere. Key padding (the SegmentIds mask at
 * attention.py:272-278 and the Hunyuan key-valid mask,
 * src/vidax/models/hunyuan_video/common/dit_layers.py:150-191) is expressed
 * as kv_len: keys at index >= kv_len[b] are invisible.
 */
typedef struct vx_attn_args {
  const void* q;  /* (B, Sq, Hq, D) bf16 */
  const void* k;  /* (B, Sk, Hkv, D) bf16 */
  const void* v;  /* (B, Sk, Hkv, D) bf16 */
  void* o;        /* (B, Sq, Hq, D) bf16 */
  int64_t q_stride[3]; /* element strides of dims (b, s, h); d stride must be 1 */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int32_t batch, seq_q, seq_k, heads_q, heads_kv, head_dim;
  float scale;             /* softmax scale, > 0 */
  const int32_t* kv_len;   /* optional device int32[B]; NULL = all seq_k keys valid;
                              kv_len[b] <= 0 writes zero rows (and lse -inf) for item b */
  float* lse;              /* optional device fp32 (B, Hq, Sq): natural-log sum-exp */
  int32_t schedule;        /* VX_SCHED_STATIC (default) or VX_SCHED_DYNAMIC */
} vx_attn_args;

/* Work distribution of vx_attn_fwd: STATIC = one CTA per SM, each taking a
 * fixed share of the (query block, head, batch) units -- best when the kernel
 * has the GPU to itself; DYNAMIC = CTAs take over not-yet-launched work at run
 * time (hardware cluster launch control) -- best when other kernels (e.g.
 * collectives) run concurrently and hold some SMs. */
enum { VX_SCHED_STATIC = 0, VX_SCHED_DYNAMIC = 1 };

int vx_attn_fwd(const vx_attn_args* args, vx_stream_t stream);

/* ----------------------------------------------------------------------
 * DeepSpeed-Ulysses head-slab packing (one batch item per call).
 *
 * Replaces the layout half of the tiled jax.lax.all_to_all calls in
 * sequence_parallel_self_attention (src/vidax/core/attention.py:379-381 and
 * :388): after vx_ulysses_pack, chunk g of `dst` (groups equal contiguous
 * chunks) holds head group g of every local token, so one equal-split
 * all-to-all (NCCL) delivers the tokens->heads reshard; the receiver's buffer
 * (groups_src, seq, hg, D) is the full sequence in source-rank order.
 * hg = ceil(heads / groups); pack writes zeros for heads >= `heads`
 * (head padding when heads % groups != 0) and unpack drops them.
 */
typedef struct vx_head_slab_args {
  int32_t num_tensors;   /* 1..3 (e.g. q, k, v in one launch) */
  const void* src[3];
  void* dst[3];
  int64_t stride[3][2];  /* strided side, element strides of (seq, heads); d stride 1 */
  int32_t seq, heads, head_dim, groups;
  /* Optional sub-group selection (all 0 = whole groups): packed head i of
   * group g is strided head head_offset + g * group_stride + i for
   * i < slab_heads; heads with i >= group_valid or index >= `heads` are
   * zero (pack) / skipped (unpack). Lets one all-to-all move a sub-group of
   * every rank's head group, so transfers can be pipelined against the
   * attention kernel. */
  int32_t slab_heads, group_stride, head_offset, group_valid;
} vx_head_slab_args;

/* strided (seq, heads, D) rows -> contiguous (groups, seq, hg, D) */
int vx_ulysses_pack(const vx_head_slab_args* args, vx_stream_t stream);
/* contiguous (groups, seq, hg, D) -> strided (seq, heads, D) rows */
int vx_ulysses_unpack(const vx_head_slab_args* args, vx_stream_t stream);

/* ----------------------------------------------------------------------
 * The Ulysses all-to-alls done by the slab kernels over NVLink: replaces
 * the tiled jax.lax.all_to_all pair of sequence_parallel_self_attention
 * (src/vidax/core/attention.py:379-381 tokens->heads, :388 heads->tokens)
 * for ranks on one NVLink / NVSwitch domain whose buffers are mapped into
 * each other's processes (vx_ipc_*).
 *
 * vx_ulysses_pack_peers is vx_ulysses_pack with group g's packed chunk
 * (seq, hg, D) stored straight to peer[t][g] -- the slot of this rank's
 * chunk in rank g's receive slab -- instead of to slab.dst: packing and the
 * tokens->heads exchange in one pass of SM stores over NVLink.
 * vx_ulysses_unpack_peers is vx_ulysses_unpack reading group g's chunk
 * straight from peer[t][g] -- this rank's tokens in rank g's attention
 * output -- into the strided rows at slab.dst: the heads->tokens exchange
 * and the unpack in one pass of loads over NVLink. Order with the other
 * ranks' work through vx_peer_barrier. */
typedef struct vx_peer_slab_args {
  vx_head_slab_args slab; /* as for vx_ulysses_pack / vx_ulysses_unpack; pack ignores slab.dst,
                             unpack ignores slab.src */
  void* peer[3][8];       /* per tensor t and group g < slab.groups (<= 8): the remote chunk */
  int32_t max_ctas;       /* CTA budget over all groups and tensors; 0 = as many as the data
                             fills. A small budget leaves SMs to a concurrent kernel. */
} vx_peer_slab_args;
int vx_ulysses_pack_peers(const vx_peer_slab_args* args, vx_stream_t stream);
int vx_ulysses_unpack_peers(const vx_peer_slab_args* args, vx_stream_t stream);

/* Barrier of `world` ranks (one GPU each) through flags in their memory:
 * each rank writes `epoch` into slot `rank` of every rank's flag array
 * (after a system-scope fence, so the peer stores of the kernels before it
 * on `stream` are visible first), then waits until every slot of its own
 * array holds at least `epoch`. Stream-ordered: later work on `stream` sees
 * what the other ranks wrote before their arrival. Each flag array is used
 * by one sequence of barriers, issued in the same order on every rank, with
 * epoch = 1, 2, ... The wait is bounded by timeout_ns (0: 2 s); on expiry
 * the kernel sets VX_DEV_TIMEOUT_PEER in the device status word
 * (vx_device_status) and returns. */
typedef struct vx_peer_barrier_args {
  uint32_t* flags[8];  /* flags[g]: rank g's array of `world` uint32 (flags[rank] is local) */
  int32_t rank, world;
  uint32_t epoch;
  int64_t timeout_ns;
} vx_peer_barrier_args;
int vx_peer_barrier(const vx_peer_barrier_args* args, vx_stream_t stream);
#define VX_DEV_TIMEOUT_PEER 32

/* CUDA IPC of device memory allocated with cudaMalloc (torch's default
 * allocator included): the 64-byte handle of the allocation holding
 * dev_ptr and dev_ptr's offset in it; another process opens the handle
 * (mapping the allocation, peer access enabled on first use) and adds the
 * offset; vx_ipc_close unmaps. */
int vx_ipc_get_handle(const void* dev_ptr, char handle_out[64], int64_t* offset_out);
int vx_ipc_open(const char handle[64], void** base_out);
int vx_ipc_close(void* base);

/* ----------------------------------------------------------------------
 * The whole DeepSpeed-Ulysses layer behind one call, over an NCCL
 * communicator: replaces sequence_parallel_self_attention
 * (src/vidax/core/attention.py:341-388) -- the tokens->heads all_to_all of
 * q, k, v (:379-381), local attention over the full sequence for this rank's
 * head group (:383-386), the heads->tokens all_to_all (:388) -- for hosts
 * without the torch mirror (vidax_b200.ulysses). The rank's head group
 * (ceil(heads / world) heads, zero heads past `heads`) is processed in
 * pipelined slices: slice j+1's exchange runs on an internal stream while
 * the attention kernel computes slice j, and slice j's reverse exchange
 * overlaps slice j+1. All work is ordered after prior work on `stream` and
 * complete before later work on it; the host does not block.
 *
 * NCCL is not linked: its entry points are looked up at run time in the
 * NCCL already loaded in the process (e.g. by torch), else libnccl.so.2.
 * A vx_comm wraps either the caller's communicator (vx_comm_wrap, e.g.
 * torch's ProcessGroupNCCL communicator; not destroyed here) or one created
 * from a unique id every rank received from rank 0 (vx_comm_init: the
 * vx_comm_* entry points of the C ABI this library proposes for a JAX host,
 * which has no NCCL communicator of its own to lend).
 */
typedef struct vx_comm vx_comm;
typedef struct vx_ulysses_args {
  const void* q;  /* (B, S_loc, H, D) bf16: this rank's tokens [r*S_loc, (r+1)*S_loc) */
  const void* k;
  const void* v;
  void* o;        /* (B, S_loc, H, D) bf16 */
  int64_t q_stride[3]; /* element strides of (b, s, h); d stride 1, multiples of 8 */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int32_t batch, seq_local, heads, head_dim;
  float scale;          /* softmax scale, > 0 */
  int32_t valid_len;    /* 0: all world * seq_local tokens are real; else keys >= valid_len are
                           padding, invisible to every query (the sequence padded to a multiple
                           of the world size) */
  void* workspace;      /* device memory, 256-byte aligned, vx_ulysses_workspace_size bytes; only
                           one call may use it at a time */
  int64_t workspace_bytes;
} vx_ulysses_args;

/* NCCL unique id (128 bytes) for vx_comm_init, made on one rank and sent to
 * every other rank by the host. */
int vx_comm_get_unique_id(char uid_out[128]);
/* Creates this rank's communicator (collective: every rank calls it, each on
 * its own GPU, current at the call). */
int vx_comm_init(int32_t rank, int32_t world, const char uid[128], vx_comm** comm_out);
/* Wraps an existing ncclComm_t of the current device (borrowed). */
int vx_comm_wrap(void* nccl_comm, vx_comm** comm_out);
/* Releases the wrapper (and the communicator if vx_comm_init made it). */
int vx_comm_destroy(vx_comm* comm);
/* Workspace bytes a call with these arguments needs on a `world`-rank axis. */
int vx_ulysses_workspace_size(const vx_ulysses_args* args, int32_t world, int64_t* bytes_out);
int vx_ulysses_attn_fwd(const vx_ulysses_args* args, vx_comm* comm, vx_stream_t stream);
/* vx_ulysses_attn_fwd for callers that may not allocate device memory: an
 * XLA custom call, for one, whose device memory belongs to XLA's allocator
 * (which reserves most of it up front), so a cudaMalloc inside the handler
 * can fail and synchronizes the device. No counterpart in the reference:
 * its JAX layer gets scratch from XLA.
 *
 * Same layer and results as vx_ulysses_attn_fwd; `workspace` and
 * `workspace_bytes` are ignored. The workspace is instead a built-in 32 MiB
 * device array (every GPU on which this library's device code is loaded
 * holds it until the process exits); a call whose vx_ulysses_workspace_size
 * exceeds 32 MiB fails with VX_EINVAL. The entry point allocates nothing.
 * The first call on a device looks the array's address up (once per device,
 * that device current); make that first call before any stream capture.
 * Every call on a device shares the array: calls that may overlap on the GPU
 * (on different streams, or from several threads) race on it, so issue them
 * in order on one stream. Nothing in it needs clearing: each call writes
 * every workspace byte it reads. */
int vx_ulysses_attn_fwd_static(const vx_ulysses_args* args, vx_comm* comm, vx_stream_t stream);

/* ----------------------------------------------------------------------
 * Fused pre-attention step: RMSNorm + 3-D RoPE + head-slab pack, one HBM
 * pass over q / k / v.
 *
 * Replaces, per layer, the sequence after the q/k/v projections in Wan's
 * attention (src/vidax/models/wan/common/dit_layers.py:137-157):
 * RMSNorm(dim) on q and k (src/vidax/core/attention.py:149-162), the reshape
 * to (B, S, H, D), apply_rope3d (src/vidax/core/rope3d.py:89-111) and the
 * tokens->heads packing of sequence_parallel_self_attention
 * (attention.py:379-381). per_head = 1 gives RMSNorm(head_dim) of
 * HunyuanVideo (hunyuan_video/common/dit_layers.py:358) and LTX-2.5's
 * neighborhood attention (ltx2_5/diffusion_vae.py:263), whose q scaling
 * (:265) is post_scale.
 *
 * Per tensor t (weight NULL: no norm; rope bit clear: no rotation; both, and
 * post_scale 1: plain pack, e.g. v):
 *   y = bf16(bf16(x * 1/sqrt(sum(x^2)/cols + eps)) * bf16(w))   cols = H*D or D
 *   y = bf16(y * post_scale)                                    if != 1
 *   (y[2p], y[2p+1]) -> (bf16(a c - b s), bf16(b c + a s)),  c, s = cos/sin[token][p]
 *
 * dst[t], per batch item b (item size groups * seq * hg * D elements,
 * hg = ceil(heads / groups)), slice by slice j:
 *   [j][g][s][i < slice_heads[j]][D]   with head = g * hg + slice_off[j] + i,
 * zero for head >= heads. groups = 1, one slice: plain (B, seq, heads, D).
 */
typedef struct vx_norm_rope_pack_args {
  int32_t num_tensors;          /* 1..3 */
  const void* src[3];           /* bf16 rows, d contiguous */
  void* dst[3];                 /* bf16, contiguous packed layout above */
  int64_t src_stride[3][3];     /* element strides of (batch, seq, head); multiples of 8 */
  const float* norm_weight[3];  /* H*D (per_head 0) or D (per_head 1) floats; NULL = no norm */
  int32_t per_head;
  float eps;
  float post_scale[3];          /* 1.0 = none */
  const float* rope_cos;        /* (seq, D/2) float tables, token-major; NULL = no RoPE */
  const float* rope_sin;
  int64_t rope_stride;          /* floats between consecutive tokens (multiple of 4, >= D/2) */
  int32_t rope_mask;            /* bit t: rotate tensor t */
  int32_t batch, seq, heads, head_dim;
  int32_t groups;               /* destination head groups (Ulysses ranks); 1 = no regrouping */
  int32_t num_slices;           /* 0 (one slice of hg heads) or 1..8 */
  int32_t slice_heads[8];       /* heads per group in each slice; sum = hg */
} vx_norm_rope_pack_args;

int vx_norm_rope_pack(const vx_norm_rope_pack_args* args, vx_stream_t stream);

/* ----------------------------------------------------------------------
 * 3-D neighborhood attention (NATTEN-style clamped windows, non-causal).
 *
 * Replaces vidax.models.ltx2_5.diffusion_vae.neighborhood_attention_3d
 * (src/vidax/models/ltx2_5/diffusion_vae.py:179-234): for query (t, h, w)
 * the keys are [st(t), st(t)+Kt) x [st(h), st(h)+Kh) x [st(w), st(w)+Kw) with
 * K = min(kernel, L) and st(i) = clamp(i - K/2, 0, L - K) (_window_start,
 * :152-164); softmax in fp32 over those keys. vidax pre-scales q by the
 * caller (:265), so `scale` is normally 1. With round_logits = 1 the q.k
 * products are rounded to bf16 before the softmax, as the reference's bf16
 * einsum does (:222).
 */
typedef struct vx_na3d_args {
  const void* q;  /* (B, T, H, W, NH, HD) bf16 */
  const void* k;  /* (B, T, H, W, NHkv, HD) bf16 */
  const void* v;
  void* o;        /* (B, T, H, W, NH, HD) bf16 */
  int64_t q_stride[5]; /* element strides of (b, t, h, w, head); d stride 1; b stride = T * t stride */
  int64_t k_stride[5];
  int64_t v_stride[5];
  int64_t o_stride[5];
  int32_t batch, T, H, W, heads, heads_kv, head_dim;
  int32_t kernel_t, kernel_h, kernel_w;
  float scale;
  int32_t round_logits;
  int32_t q_box[3];    /* query tile box (t, h, w), product 128; all 0 = choose automatically */
  int32_t pair_axis;   /* 0-2: a CTA pairs two query boxes adjacent along t / h / w; 3: it
                          pairs heads h and h + 1 of one box (head_dim 64 only); ignored when
                          q_box is 0 (the library picks box and pairing by a time model) */
  int32_t kv_tile[3];  /* key tile box (t, h, w) with q_box: all 0 = (2, 4, 16); head pairs also
                          take (4, 2, 16), (2, 8, 8) and (4, 4, 8) */
} vx_na3d_args;

int vx_na3d_fwd(const vx_na3d_args* args, vx_stream_t stream);

/* The tiling vx_na3d_fwd picks for a T x H x W grid and window (q_box all 0):
 * query box, pairing (0-2 box pairs along t / h / w, 3 head pairs) and key
 * tile, from the library's time model. Host only (no device work); for
 * inspection and tuning. No counterpart in the reference (its NA is one
 * einsum over gathered windows). */
int vx_na3d_tiling(int32_t T, int32_t H, int32_t W, int32_t kernel_t, int32_t kernel_h,
                   int32_t kernel_w, int32_t head_dim, int32_t q_box_out[3], int32_t* pair_out,
                   int32_t kv_tile_out[3]);

/* Time-slab form of vx_na3d_fwd for sequence (T-axis) sharding: q and o hold
 * frames [q_t0, q_t0 + T) of a T_global-frame grid, k and v frames
 * [kv_t0, kv_t0 + T_kv) (the caller's own frames plus the halo received from
 * the ranks that own its neighbours); windows are clamped to the global grid
 * exactly as in the unsharded call. The key frames must cover every window of
 * the slab's queries, else VX_EINVAL. k / v strides describe the T_kv-frame
 * buffers. No reference counterpart as a function: vidax shards the
 * neighborhood attention of ltx2_5/diffusion_vae.py by heads only; this is
 * the T-slab alternative of its multi-device layouts. */
typedef struct vx_na3d_slab {
  int32_t T_global;
  int32_t q_t0;
  int32_t kv_t0;
  int32_t T_kv;
} vx_na3d_slab;

int vx_na3d_fwd_slab(const vx_na3d_args* args, const vx_na3d_slab* slab, vx_stream_t stream);

/* Host helper: start_out[i] = clamp(i - K/2, 0, length - K), K = min(kernel,
 * length), i in [0, length) -- the window-start contract of _window_start
 * (diffusion_vae.py:152-164). Returns VX_EINVAL for length/kernel < 1. */
int vx_na3d_window_start(int32_t length, int32_t kernel, int32_t* start_out);

/* ----------------------------------------------------------------------
 * Strided row copy (host <-> device or device <-> device), stream-ordered:
 * `rows` rows of `row_bytes` bytes from src (pitch src_pitch) to dst (pitch
 * dst_pitch). Used by the host-buffer attention path to move one head group
 * of a BSHD tensor (a 2-D strided slab) while other groups compute; host
 * memory must be page-locked for the copy to overlap.
 */
int vx_memcpy_rows_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                         int64_t row_bytes, int64_t rows, vx_stream_t stream);

/* ----------------------------------------------------------------------
 * Fused elementwise glue of the DiT block (no counterpart in vidax's FFI
 * surface: these replace chains of framework ops around the sub-layers of
 * WanDiTBlock, src/vidax/models/wan/wan2_1/dit.py:100-156).
 *
 * vx_ln_modulate: y = bf16(((x - mean) * rsqrt(var + eps) [* w + b])
 *                          * (1 + scale[batch]) + shift[batch])
 * per row of x (rows, dim) float32, statistics as flax's LayerNorm
 * (var = E[x^2] - E[x]^2); w / b (dim) and scale / shift (rows /
 * rows_per_batch, dim) are optional (NULL; scale and shift together). dim a
 * multiple of 4, pointers 16-byte aligned.
 *
 * vx_gated_residual: x += float(y) * gate[batch] (gate NULL: x += y), x
 * float32 and y bf16 of (rows, dim), gate (rows / rows_per_batch, dim); dim
 * a multiple of 8, pointers 32-byte (x) / 16-byte (y, gate) aligned.
 */
int vx_ln_modulate(const float* x, void* y, const float* w, const float* b, const float* scale,
                   const float* shift, int64_t rows, int32_t dim, int32_t rows_per_batch,
                   float eps, vx_stream_t stream);
int vx_gated_residual(float* x, const void* y, const float* gate, int64_t rows, int32_t dim,
                      int32_t rows_per_batch, vx_stream_t stream);

/* Self-test of the bounded-wait machinery (failure detection without a GPU
 * fault): runs one CTA that waits on an mbarrier nothing arrives on, through
 * the same bounded wait the kernels use, with a limit of `limit_cycles` SM
 * cycles. The wait gives up, raises the CTA's abort flag and records status
 * bit 16 in the device status word; returns VX_ETIMEOUT with *status_out set
 * to the status word (VX_ECUDA if the wait did not behave as specified). The
 * context stays usable; clear the word with vx_device_status(.., 1).
 * All calls on a device share one file-scope 2-int __device__ array for the
 * wait's report: calls that overlap (e.g. from two host threads) race on it
 * and must be serialised by the caller. *status_out is the whole status word,
 * so it may also carry bits that other kernels running meanwhile set. */
int vx_selftest_wait_timeout(int64_t limit_cycles, int* status_out);

#ifdef __cplusplus
}
#endif

#endif /* VIDAX_CUDA_H_ */
