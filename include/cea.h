/*
 * cea.h — C ABI of the B200 sequence-parallel attention library (libcea.so).
 *
 * The library implements the compute of collab_infer's sequence-parallel
 * attention path on sm_100a.  Every entry point takes plain pointers, sizes
 * and strides (in elements), enqueues work on the given CUDA stream, never
 * synchronises the host and never allocates: buffers, including workspaces,
 * belong to the caller.  Functions return CEA_OK (0) or a positive error
 * code; cea_last_error() gives the thread's last message.
 *
 * Tensor conventions (as in collab_infer):
 *   q [B, Sq, Hq, D], k/v [B, Sk, Hkv, D], out [B, Sq, Hq, D]: token-major,
 *     any strides for (b, s, h), the D axis contiguous;
 *   lse [B, Hq, Sq] natural-log log-sum-exp, any strides;
 *   positions [B, S] int64, -1 = padding; key j is visible to query i iff
 *     k_pos[j] >= 0 && (!causal || k_pos[j] <= q_pos[i]);
 *   rows with no visible key give out = 0 and lse = -inf.
 */
#ifndef CEA_H_
#define CEA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CEA_ABI_VERSION 7

enum cea_status {
  CEA_OK = 0,
  CEA_ERR_INVALID = 1,     /* bad argument (shapes, strides, null pointers) */
  CEA_ERR_UNSUPPORTED = 2, /* dtype / shape combination without a kernel */
  CEA_ERR_CUDA = 3,        /* CUDA runtime or driver error */
  CEA_ERR_WORKSPACE = 4,   /* workspace missing or too small */
  CEA_ERR_DEVICE = 5,      /* a kernel reported a device-side error (see cea_device_status) */
  CEA_ERR_NCCL = 6         /* NCCL library missing, or an NCCL call failed */
};

/* device-side error codes stored by kernels (bounded waits that expired) */
enum cea_device_error {
  CEA_DEV_OK = 0,
  CEA_DEV_TIMEOUT_PRODUCER = 0x101,
  CEA_DEV_TIMEOUT_MMA = 0x102,
  CEA_DEV_TIMEOUT_SOFTMAX = 0x103,
  CEA_DEV_TIMEOUT_DECODE = 0x104,
  CEA_DEV_TIMEOUT_PEER = 0x105
};

typedef enum cea_dtype { CEA_F32 = 0, CEA_F16 = 1, CEA_BF16 = 2, CEA_F64 = 3 } cea_dtype;

/*
 * Attention with log-sum-exp over position-masked keys.
 *
 * Replaces collab_infer parallel/attention.py:201-239 (attention_with_lse),
 * :270-301 (attention, lse == NULL) and, with accumulate = 1, the pairwise
 * merge of :242-250 fused into the epilogue (the ring-attention step of
 * parallel/sequence_parallel.py:117-121).
 *
 * in_dtype: q/k/v dtype.  out_dtype: dtype of out (F32 or F64 for the
 * accumulation precision of attention_with_lse, or the input dtype for
 * attention).  lse has dtype F64 when in_dtype is F64, else F32.
 * accumulate = 1 merges the result into the (out, lse) already stored
 * (requires lse and an F32/F64 out).
 * kv_map (optional, length Hq, int32): KV head of every query head; NULL means
 * query head h uses KV head h / (Hq / Hkv).
 */
typedef struct cea_attn_params {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  void* lse;
  const int64_t* q_pos;
  const int64_t* k_pos;
  const int32_t* kv_map;
  int64_t q_stride[3];   /* b, s, h */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t lse_stride[3]; /* b, h, s */
  int64_t qpos_stride[2]; /* b, s */
  int64_t kpos_stride[2];
  int32_t B, Sq, Sk, Hq, Hkv, D;
  double scale;
  int32_t causal;
  int32_t in_dtype;
  int32_t out_dtype;
  int32_t accumulate;
  void* workspace;
  size_t workspace_bytes;
  /* Optional decode-step cache append, served by the split-KV decode path only (cea_attn_kernel_kind 2;
   * other paths fail with CEA_ERR_UNSUPPORTED).  The last n_new of the Sk keys are this step's new
   * tokens: the kernel reads their K, V and positions from new_k / new_v ([B, n_new, Hkv, D], element
   * strides b, s, h; D contiguous, rows 16-byte aligned) and new_pos ([B, n_new]) and writes them into the
   * last n_new rows of k, v and k_pos, which must therefore be writable (the caller's KV-cache views).
   * This replaces the separate append launch before the decode (collab_infer models/cache.py:51-62,
   * engine/engine.py:239-243).  n_new = 0 (zero-initialised) disables it. */
  const void* new_k;
  const void* new_v;
  const int64_t* new_pos;
  int64_t new_k_stride[3];
  int64_t new_v_stride[3];
  int64_t new_pos_stride[2];
  int32_t n_new;
  /* Optional source of the running result for accumulate = 1 with a 16-bit out, served by the tcgen05
   * prefill path only (cea_attn_kernel_kind 1; other paths fail with CEA_ERR_UNSUPPORTED).  The stored
   * result is read from acc_in ([B, Sq, Hq, D] F32, element strides b, s, h; rows 16-byte aligned)
   * instead of out, merged with this call's partial, and written to out in the input dtype; lse is
   * updated in place.  This fuses the last ring step's merge with the final cast to the activation
   * dtype (collab_infer parallel/sequence_parallel.py:117-130).  NULL (zero-initialised) disables it. */
  const float* acc_in;
  int64_t acc_stride[3];
} cea_attn_params;

/* Bytes of workspace cea_attn_fwd needs for these parameters (0 if none). */
size_t cea_attn_workspace_size(const cea_attn_params* p);

/* Kernel cea_attn_fwd would run: 0 none (empty), 1 tcgen05 prefill, 2 split-KV decode, 3 SIMT. */
int cea_attn_kernel_kind(const cea_attn_params* p);

int cea_attn_fwd(const cea_attn_params* p, void* stream);

/*
 * Split-KV decode (few query rows per KV head against a long KV cache).
 * Replaces the local attention of collab_infer parallel/sequence_parallel.py:270-272
 * (distributed_kv_attention).  Same parameters as cea_attn_fwd; requires
 * Sq * (Hq / Hkv) <= 16, uniform groups (kv_map NULL), bf16/f16, D in {64, 128}.
 * The workspace holds the per-split partial results.
 */
int cea_decode_splitkv(const cea_attn_params* p, void* stream);

/*
 * Split-KV decode that allocates nothing.  It has no counterpart in the
 * reference: collab_infer's decode always allocates its partial results.
 *
 * Same parameters and result as cea_decode_splitkv, but p->workspace is
 * ignored.  The per-split partials go to a fixed device array inside the
 * library instead.  That array is CEA_NOALLOC_SCRATCH_BYTES on every GPU that
 * loads libcea.so and is held until the process exits.  This entry point is
 * meant for callers that only hold the input and output buffers and have no
 * allocator to size a workspace from, such as a serving loop that reserves all
 * its device memory at start-up and treats any later allocation as an error.
 *
 * The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  The address is kept per device and looked up
 * again when the device's current CUDA context changes (after a device reset
 * the module, and the array with it, is loaded into a new context); the array's
 * contents do not survive that.  Calls share the array, so calls that overlap on
 * the GPU (for example on two streams) race and must be ordered by the caller.
 * The split count is reduced to fit the array (e.g. B=128, Hq=16, D=128,
 * Sq=1: 1.06 MB per split, at most 7 splits where the regular plan may use
 * more).  A call whose single split of partials, B*Hq*Sq*(D+1)*4 bytes,
 * exceeds it fails with CEA_ERR_WORKSPACE.
 * It never calls cudaMalloc or cudaFree.
 */
#define CEA_NOALLOC_SCRATCH_BYTES (8u << 20)
int cea_decode_splitkv_noalloc(const cea_attn_params* p, void* stream);

/*
 * Exact merge of n partial attention results over disjoint key sets.
 * Replaces collab_infer parallel/attention.py:242-264 (merge_attention,
 * merge_attention_list).  Partial i is (outs[i], lses[i]); all partials share
 * the strides below.  out may alias outs[0] / lse may alias lses[0].
 */
#define CEA_MAX_MERGE 32
typedef struct cea_merge_params {
  int32_t n;
  const void* outs[CEA_MAX_MERGE];
  const void* lses[CEA_MAX_MERGE];
  void* out;
  void* lse; /* may be NULL */
  int64_t part_o_stride[3];   /* b, s, h */
  int64_t part_lse_stride[3]; /* b, h, s */
  int64_t o_stride[3];
  int64_t lse_stride[3];
  int32_t B, Sq, H, D;
  int32_t part_dtype; /* F32 or F64 (partials and lse) */
  int32_t out_dtype;  /* F32, F64, BF16 or F16 */
} cea_merge_params;

int cea_merge(const cea_merge_params* p, void* stream);

/*
 * Segment copy for the Ulysses all-to-all (collab_infer
 * parallel/sequence_parallel.py:163-177 and :191-194): segment i copies the
 * [nb, ns, nh, D] block at src (strides src_stride, elements) to dst
 * (strides dst_stride).  Used to pack per-peer head slices of q/k/v into one
 * send buffer, to lay received blocks out as the full sequence and to put the
 * returned head blocks back into [B, s, H, D].
 */
#define CEA_MAX_SEGMENTS 64
typedef struct cea_segment {
  const void* src;
  void* dst;
  int64_t src_stride[3]; /* b, s, h */
  int64_t dst_stride[3];
  int32_t nb, ns, nh;
} cea_segment;

typedef struct cea_copy_params {
  int32_t n;
  int32_t D;
  int32_t elem_bytes; /* 2, 4 or 8 */
  cea_segment seg[CEA_MAX_SEGMENTS];
} cea_copy_params;

int cea_ulysses_pack(const cea_copy_params* p, void* stream);
int cea_ulysses_unpack(const cea_copy_params* p, void* stream);

/*
 * Ring wire pack / unpack (collab_infer parallel/sequence_parallel.py:101-103
 * and :129, over Communicator.to_wire, distributed/comm.py:275-290): two
 * [B, S, H, D] tensors (K and V; element strides b, s, h per tensor, D
 * contiguous) copied into two destinations with a dtype conversion in the
 * same pass.  Packing writes the K||V message of a ring step in the wire
 * dtype; unpacking widens a received message back to the compute dtype.
 * Conversions follow torch: float64 goes through float32, narrowing rounds
 * to nearest even, and a float16 destination saturates at +-65504 (NaN is
 * kept) unless the source is float16 too.
 */
typedef struct cea_wire_cast_params {
  const void* src[2];
  void* dst[2];
  int64_t src_stride[2][3];
  int64_t dst_stride[2][3];
  int32_t B, S, H, D;
  int32_t src_dtype, dst_dtype; /* cea_dtype */
} cea_wire_cast_params;

int cea_wire_cast(const cea_wire_cast_params* p, void* stream);

/*
 * The decoder-layer steps around the attention for a LLaMA-family prefill
 * or decode on the sequence-parallel path (collab_infer models/llama.py).
 * Values are rounded to the model dtype wherever the reference's tensor
 * expressions round them.
 *
 * cea_add_rmsnorm: resid <- resid + delta (if delta != NULL), then
 *   y = w * (resid * rsqrt(mean(resid^2) + eps)) over the last dimension h,
 *   the normalisation in fp32 (fp64 for an fp64 model); RMSNorm.forward,
 *   llama.py:52-61, fused with the residual adds of DecoderLayer.forward,
 *   :337-339.  Rows are contiguous; strides count elements between rows.
 */
typedef struct cea_rmsnorm_params {
  void* resid;
  const void* delta;
  const void* weight;
  void* y;
  int64_t rows, h;
  int64_t resid_stride, delta_stride, y_stride;
  double eps;
  int32_t dtype;
} cea_rmsnorm_params;

int cea_add_rmsnorm(const cea_rmsnorm_params* p, void* stream);

/*
 * cea_rope: in place, x <- x * cos + rotate_half(x) * sin for q
 * [B, S, Hq, D] and k [B, S, Hk, D] (element strides b, s, h; D contiguous)
 * with cos / sin of max(pos, 0) * inv_freq (RotaryEmbedding and
 * apply_rotary, llama.py:64-88).  inv_freq holds D/2 floats (doubles for an
 * fp64 model); pos is [B, S] int64.
 */
typedef struct cea_rope_params {
  void* q;
  void* k;
  int64_t q_stride[3];
  int64_t k_stride[3];
  const int64_t* pos;
  int64_t pos_stride[2];
  const void* inv_freq;
  int32_t B, S, Hq, Hk, D;
  int32_t dtype;
} cea_rope_params;

int cea_rope(const cea_rope_params* p, void* stream);

/*
 * cea_silu_mul: out = silu(gate) * up for rows of n units (ParallelMLP,
 * llama.py:301-305); gate and up rows are in_stride elements apart (the two
 * halves of the fused gate/up projection).
 */
typedef struct cea_silu_mul_params {
  const void* gate;
  const void* up;
  void* out;
  int64_t rows, n;
  int64_t in_stride, out_stride;
  int32_t dtype;
} cea_silu_mul_params;

int cea_silu_mul(const cea_silu_mul_params* p, void* stream);

/*
 * KV-cache append (collab_infer models/cache.py:51-62, LayerKVCache.append):
 * copies n new tokens of token-major k [B, n, Hk, Dk] and v [B, n, Hv, Dv]
 * into the head-major cache buffers [B, Hk, capacity, Dk] and
 * [B, Hv, capacity, Dv] at token slots offset .. offset + n - 1, and their
 * positions [B, n] (int64) into the cache's positions [B, capacity], in one
 * launch.  The same call moves the cached tokens into a grown buffer
 * (cache.py:39-49: source = the old cache seen token-major, offset 0).
 * Strides are in elements; the innermost (D) dimension is contiguous.  k and
 * v are copied bit for bit (any dtype of 1, 2, 4 or 8 bytes); pos and
 * pos_cache are both NULL to leave positions alone.  The ring-mode decode
 * owner (engine/engine.py:235-244) is host logic and stays in the caller.
 */
typedef struct cea_kv_append_params {
  const void* k;
  const void* v;
  void* k_cache;
  void* v_cache;
  int64_t k_stride[3];  /* source b, s, h */
  int64_t v_stride[3];
  int64_t kc_stride[3]; /* cache b, t, h */
  int64_t vc_stride[3];
  const int64_t* pos;
  int64_t pos_stride[2]; /* source b, s */
  int64_t* pos_cache;
  int64_t pc_stride[2]; /* cache b, t */
  int32_t B, n, Hk, Dk, Hv, Dv;
  int32_t k_elem_bytes, v_elem_bytes;
  int64_t offset, capacity;
} cea_kv_append_params;

int cea_kv_append(const cea_kv_append_params* p, void* stream);

/*
 * NCCL transfers of the sequence-parallel path, for callers that hold no
 * PyTorch process group.  They stand in for collab_infer's Communicator
 * (distributed/comm.py:200) and its set-up:
 *   cea_nccl_get_unique_id / cea_nccl_comm_init  - process-group creation
 *     (init_distributed, distributed/launcher.py:55-97; the per-axis
 *     Communicators of distributed/mesh.py:89-110);
 *   cea_nccl_comm_destroy / cea_nccl_abort       - teardown;
 *   cea_ring_step  - the grouped send to r+1 / receive from r-1 of one ring
 *     attention step (parallel/sequence_parallel.py:108-116 over
 *     Communicator.isend/irecv, comm.py:574-610);
 *   cea_alltoallv  - the uneven all-to-all of ulysses_scatter/gather
 *     (sequence_parallel.py:163-194, Communicator.all_to_all, comm.py:468-524);
 *   cea_allgather  - the all-gather of distributed_kv_attention and
 *     gather_sequence (sequence_parallel.py:50-62,270-276,
 *     Communicator.all_gather_list, comm.py:369-410).
 * NCCL is loaded at run time: CEA_NCCL_LIBRARY if set, else the libnccl.so.2
 * already loaded in the process, else libnccl.so.2 from the loader path.
 * Buffers are device memory of the communicator's GPU, sizes in bytes; the
 * transfers are enqueued on `stream` and never synchronise the host.
 * cea_nccl_comm_init binds the communicator to the current CUDA device and,
 * like every NCCL initialisation, blocks until all ranks have called it.
 */
#define CEA_NCCL_ID_BYTES 128
typedef struct cea_nccl_comm cea_nccl_comm;

/* A fresh NCCL unique id (CEA_NCCL_ID_BYTES bytes) for rank 0 to hand to the others. */
int cea_nccl_get_unique_id(void* id_out);
int cea_nccl_comm_init(cea_nccl_comm** comm_out, int rank, int nranks, const void* id);
int cea_nccl_comm_destroy(cea_nccl_comm* comm);
/* Aborts outstanding NCCL work of the communicator and frees it (error paths). */
int cea_nccl_abort(cea_nccl_comm* comm);
/* Sends send_bytes to rank `to` and receives recv_bytes from rank `from`, as one NCCL group. */
int cea_ring_step(cea_nccl_comm* comm, const void* send, size_t send_bytes, int to, void* recv, size_t recv_bytes,
                  int from, void* stream);
/* Uneven all-to-all: nranks-entry arrays of byte counts and byte offsets into send / recv. */
int cea_alltoallv(cea_nccl_comm* comm, const void* send, const size_t* send_bytes, const size_t* send_offsets,
                  void* recv, const size_t* recv_bytes, const size_t* recv_offsets, void* stream);
/* recv (nranks * bytes) receives every rank's `bytes` bytes in rank order. */
int cea_allgather(cea_nccl_comm* comm, const void* send, void* recv, size_t bytes, void* stream);

/*
 * Distributed-KV decode exchange over peer memory: the all-gather of the
 * per-rank partials and their exact merge in one kernel, replacing the
 * all-gather + list merge of collab_infer parallel/sequence_parallel.py:270-276
 * (distributed_kv_attention) for ranks of one node (NVLink P2P).
 *
 * Every rank owns a receive buffer of 2 x nranks slots of rows * W floats (a
 * row: partial output in columns [0, D), its natural-log lse in column D,
 * padding; W a multiple of 4 greater than D) and nranks uint64 counters set to
 * zero, and maps every peer's buffer and counters into its address space
 * (cea_ipc_export / cea_ipc_open).  Call number `epoch` (1, 2, ... on these
 * buffers, the same on every rank) uses slot parity epoch & 1: the caller
 * first writes its own partial into slot [epoch & 1][rank] of its own buffer
 * (cea_attn_fwd or cea_decode_splitkv with out / lse pointing there), then
 * calls cea_peer_merge, which stores that slot into every peer's buffer,
 * signals every peer through its counters, waits (bounded) for every peer's
 * data and writes the merged [B, Sq, H, D] output.  Every rank must make the
 * same sequence of calls.  A wait that expires (after wait_limit_ns, or the
 * built-in 2 s when it is 0) records CEA_DEV_TIMEOUT_PEER in the device error
 * word and, when fault_flag is set, in *fault_flag (a store the host can read
 * without synchronising when it points to mapped pinned host memory), and the
 * rows the timed-out CTAs own are written as NaN.  After a timeout the
 * buffers' call numbering is no longer shared by the ranks: do not call again
 * on them.
 */
#define CEA_MAX_PEERS 16
typedef struct cea_peer_merge_params {
  int32_t n, rank;
  float* bufs[CEA_MAX_PEERS];      /* rank q's receive buffer as mapped in this process */
  uint64_t* flags[CEA_MAX_PEERS];  /* rank q's nranks counters as mapped in this process */
  uint64_t epoch;
  int32_t B, Sq, H, D, W;
  void* out;
  int64_t o_stride[3]; /* b, s, h */
  int32_t out_dtype;   /* F32, BF16 or F16 */
  int32_t* fault_flag;    /* optional: set to CEA_DEV_TIMEOUT_PEER on a timeout (device-visible address) */
  uint64_t wait_limit_ns; /* bound of the wait for the peers; 0 = the built-in 2 s */
} cea_peer_merge_params;

int cea_peer_merge(const cea_peer_merge_params* p, void* stream);

/* CUDA IPC of device memory between the processes of one node: the 64-byte
 * handle of the allocation holding `ptr`, and ptr's offset in it. */
#define CEA_IPC_HANDLE_BYTES 64
int cea_ipc_export(const void* ptr, void* handle_out, size_t* offset_out);
/* Maps a peer's allocation on the current device; *ptr_out = base + offset, *base_out for cea_ipc_close. */
int cea_ipc_open(const void* handle, size_t offset, void** ptr_out, void** base_out);
int cea_ipc_close(void* base);

/* Reads (and with clear != 0 resets) the device error word of the current device. Synchronises `stream`. */
int cea_device_status(int* status_out, int clear, void* stream);

const char* cea_last_error(void);
int cea_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CEA_H_ */
