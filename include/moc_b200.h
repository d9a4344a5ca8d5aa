/*
 * moc_b200.h — C ABI of the B200 (sm_100a) Mixture-of-Convolutions kernels.
 *
 * Every entry point takes caller-owned device pointers, plain sizes and a
 * cudaStream_t passed as `void*` (NULL = legacy default stream).  Nothing here
 * allocates device memory or synchronises the host; work is stream ordered.
 * Each call returns MOC_OK (0) or one of the MOC_ERR_* codes below;
 * moc_error_string() turns a code into text.
 *
 * Tensor layouts (all row major, innermost dimension contiguous):
 *   x, out, dy, dx          [n_tokens, dim]        (fixed length: n_tokens = batch*seq_len,
 *                                                   token row = b*seq_len + t)
 *   alpha, dalpha           [n_tokens, n_bases]
 *   basis, dbasis           [n_bases, kernel_size, dim]
 *   z, dz                   [n_tokens, z_dim]
 *   router weight, dweight  [n_bases, z_dim]
 *   decode cache            [batch, dim, kernel_size] with explicit strides
 *
 * Convolution convention (matches the reference's moc/kernels.py:99-130 and
 * moc/reference.py:28-32): tap s multiplies token t-(S-1-s), so tap S-1 is the
 * current token; taps that fall before the start of the token's sequence read 0.
 */
#ifndef MOC_B200_H
#define MOC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* floating point storage types */
#define MOC_DTYPE_F32 0
#define MOC_DTYPE_F16 1
#define MOC_DTYPE_BF16 2
/* integer index types (cu_seqlens, chunk_indices) */
#define MOC_INDEX_I32 0
#define MOC_INDEX_I64 1

/* return codes */
#define MOC_OK 0
#define MOC_ERR_INVALID_ARGUMENT 1
#define MOC_ERR_UNSUPPORTED_DTYPE 2
#define MOC_ERR_UNSUPPORTED_SHAPE 3
#define MOC_ERR_MISALIGNED 4
#define MOC_ERR_WORKSPACE_TOO_SMALL 5
#define MOC_ERR_CUDA 6
#define MOC_ERR_SCRATCH_LIMIT 7

/* Shape and routing of one convolution problem.
 * Fixed length: batch > 0, seq_len > 0, n_tokens = batch*seq_len, varlen fields zero/NULL.
 * Packed varlen: batch = seq_len = 0; cu_seqlens has n_seqs+1 monotone offsets into the
 * n_tokens rows; chunk_indices holds n_chunks (seq_id, chunk_in_seq) pairs, each covering
 * chunk_size tokens of that sequence (the reference's prepare_chunk_indices format,
 * moc/ops.py:47-104).  Only the listed chunks are computed. */
typedef struct moc_problem {
  int64_t batch;
  int64_t seq_len;
  int64_t n_tokens;
  int64_t dim;
  int32_t n_bases;
  int32_t kernel_size;
  int32_t x_dtype;     /* MOC_DTYPE_F32 or MOC_DTYPE_BF16: selects fp32 or bf16 compute */
  int32_t alpha_dtype; /* any MOC_DTYPE_* */
  int32_t basis_dtype; /* any MOC_DTYPE_* */
  int32_t activation;  /* 0 = none, 1 = SiLU applied to the convolution output */
  const void* cu_seqlens;
  int32_t cu_seqlens_dtype;
  int64_t n_seqs;
  const void* chunk_indices;
  int32_t chunk_indices_dtype;
  int64_t n_chunks;
  int32_t chunk_size;
  /* Optional, fixed length only: the conv cache [batch, dim, kernel_size] (x's dtype,
   * element strides halo_strides) of the tokens before each sequence.  The taps of the
   * first kernel_size - 1 positions then read those tokens (slot S-1 newest) instead of
   * zeros, which is prefill with a cache (the reference prepends the cache with zero
   * routing weights, moc/api.py:299-309).  The cache itself gets no gradient. */
  const void* halo;
  int64_t halo_strides[3];
} moc_problem;

/* Library identification, e.g. "moc_b200 0.1.0 sm_100a". */
const char* moc_version(void);
/* Static text for a MOC_* return code. */
const char* moc_error_string(int code);
/* Text of the last CUDA error seen by the library on this host thread (or ""). */
const char* moc_last_cuda_error(void);

/* Number of kernels this library has launched in this process (all devices, all
 * streams); lets a caller count launches over a region of work. */
uint64_t moc_launch_count(void);

/* Device status word of the TMA-staged kernels and of the fused decode step, OR of
 * MOC_STATUS_* bits recorded since the last clear (synchronous: reads device memory).  A
 * staging wait, or a wait of the decode step for another CTA's data, that runs out of its
 * poll budget records MOC_STATUS_WAIT_TIMEOUT and the kernel returns without writing its
 * outputs instead of hanging. */
#define MOC_STATUS_WAIT_TIMEOUT 1
int moc_device_status(int* status, int clear);

/* Diagnostic: launches one thread that waits, with `poll_limit` polls, on an mbarrier
 * nothing arrives on; it records MOC_STATUS_WAIT_TIMEOUT through the same path as the
 * staging kernels.  Used by the tests of the bounded-wait path. */
int moc_wait_timeout_probe(uint32_t poll_limit, void* stream);

/* Diagnostic: launches a cluster of two CTAs in which CTA 0 waits, with `poll_limit`
 * polls and the fused decode step's cross-CTA wait, for bytes that CTA 1 never sends; it
 * records MOC_STATUS_WAIT_TIMEOUT through the decode step's path and both CTAs leave
 * through the cluster's exit barrier.  Used by the tests of the bounded-wait path. */
int moc_cluster_wait_timeout_probe(uint32_t poll_limit, void* stream);

/* Kernel family selection for every later call in this process: MOC_PATH_AUTO (tensor
 * cores for the bf16 shapes they support, the default; the convolution backward of 17..32
 * bases with 5..8 taps takes its tcgen05 kernel), MOC_PATH_GENERIC (the fp32 CUDA-core
 * kernels for every shape) or MOC_PATH_WARP_BACKWARD (as AUTO, but every tensor-core
 * convolution backward takes the warp-level kernel).  All compute the complete result; the
 * switch exists so the families can be cross-checked through this ABI. */
#define MOC_PATH_AUTO 0
#define MOC_PATH_GENERIC 1
#define MOC_PATH_WARP_BACKWARD 2
int moc_set_kernel_path(int path);

/* Forward convolution: out = [silu](conv(x, alpha, basis)), out has x's dtype.
 * Replaces launch_forward / launch_preact, moc/ops.py:129-194 and 197-213
 * (launch_preact is this call with activation = 0). */
int moc_forward(const moc_problem* p, const void* x, const void* alpha, const void* basis,
                void* out, void* stream);

/* Bytes of scratch memory moc_backward needs for problem p.  The workspace passed to
 * moc_backward must start on a 16-byte boundary (MOC_ERR_MISALIGNED otherwise). */
size_t moc_backward_workspace_bytes(const moc_problem* p);

/* Backward convolution.  dy is the gradient of out.  With activation = 1 the
 * pre-activation is recomputed on chip.  Writes dx (x dtype; pass NULL to skip, the
 * reference's need_x = False), dalpha (alpha dtype) and dbasis (basis dtype).
 * dbasis is reduced deterministically (fixed-order two-pass sum, no atomics).
 * Replaces launch_backward, moc/ops.py:216-338. */
int moc_backward(const moc_problem* p, const void* x, const void* alpha, const void* basis,
                 const void* dy, void* dx, void* dalpha, void* dbasis,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Single-token decode step against the conv cache.  x [batch, dim], alpha
 * [batch, n_bases], basis [n_bases, kernel_size, dim]; cache [batch, dim, kernel_size]
 * is addressed through cache_strides (in elements) and updated in place: slots 1..S-1
 * shift to 0..S-2 and x is written to slot S-1.  out [batch, dim] has x's dtype.
 * Replaces launch_update, moc/ops.py:341-362 (kernel moc/kernels.py:442-550). */
int moc_step(int64_t batch, int64_t dim, int32_t n_bases, int32_t kernel_size,
             int32_t x_dtype, int32_t alpha_dtype, int32_t basis_dtype, int32_t activation,
             const void* x, const void* alpha, const void* basis,
             void* cache, const int64_t cache_strides[3], void* out, void* stream);

/* Router forward: alpha = act(z @ weight^T), act = softmax over n_bases (router_act 0)
 * or exp (router_act 1).  z [n_tokens, z_dim], weight [n_bases, z_dim], alpha
 * [n_tokens, n_bases]; all three share one dtype (f32, f16 or bf16); logits stay in fp32.
 * Replaces the router in MoC.forward, moc/api.py:383-388 (F.linear + softmax/exp). */
int moc_router_forward(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype,
                       int32_t router_act, const void* z, const void* weight, void* alpha,
                       void* stream);

/* Bytes of scratch memory moc_router_backward needs.  The workspace must start on a
 * 16-byte boundary when dweight is requested (MOC_ERR_MISALIGNED otherwise). */
size_t moc_router_backward_workspace_bytes(int64_t n_tokens, int64_t z_dim, int32_t n_bases,
                                           int32_t dtype);

/* Router backward from dalpha: dlogits = softmax/exp Jacobian applied to dalpha,
 * dz = dlogits @ weight (pass NULL to skip), dweight = dlogits^T @ z (pass NULL to skip;
 * reduced deterministically).  alpha is the forward output.  dalpha may have any
 * float dtype; z, weight, alpha, dz and dweight share `dtype`.
 * Replaces PyTorch autograd of moc/api.py:383-388. */
int moc_router_backward(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype,
                        int32_t router_act, const void* z, const void* weight,
                        const void* alpha, const void* dalpha, int32_t dalpha_dtype,
                        void* dz, void* dweight, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Router backward that allocates nothing, for callers that cannot call cudaMalloc (or
 * hand this library any allocator): hosts that reach the kernels only through this C ABI
 * with tensors they do not own, or code that must not allocate once it is running, such
 * as a server that plans all device memory at start-up.  Same arguments and results as
 * moc_router_backward for bf16 problems the tensor-core path supports (n_bases % 8 == 0,
 * n_bases <= 32, z_dim % 8 == 0), without the workspace: the per-CTA dweight partials go
 * to a fixed MOC_NOALLOC_SCRATCH_BYTES array in the library's device memory, which every
 * GPU that loads the library holds until the process exits.  Problems whose partials do
 * not fit return MOC_ERR_SCRATCH_LIMIT; other shapes and dtypes return
 * MOC_ERR_UNSUPPORTED_SHAPE / MOC_ERR_UNSUPPORTED_DTYPE.  The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) and keeps it for the life of the
 * process, so make that first call before any stream capture on that device; the kept
 * address does not survive cudaDeviceReset (which also frees every other allocation of
 * the process), so do not call this after a reset.  All calls share the one array: calls
 * that can overlap on the GPU (different streams, or different host threads) race on it
 * and must be serialised by the caller.  Nothing in it needs to start at zero: every CTA
 * writes its partial before the reduction reads it, and a CTA whose staging wait runs out
 * (MOC_STATUS_WAIT_TIMEOUT, see moc_device_status) writes its partial as NaN, so dweight
 * then comes out NaN instead of mixing in an earlier call's values.  No counterpart in the
 * reference (its router backward is PyTorch autograd, which allocates through the caching
 * allocator). */
#define MOC_NOALLOC_SCRATCH_BYTES (8u << 20)
int moc_router_backward_noalloc(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype,
                                int32_t router_act, const void* z, const void* weight,
                                const void* alpha, const void* dalpha, int32_t dalpha_dtype,
                                void* dz, void* dweight, void* stream);

/* Device-side chunk index builder for packed varlen (no host sync): fills
 * chunk_indices [n_chunks, 2] int32 with (seq_id, chunk_in_seq) for every
 * chunk_size-token chunk of every sequence, in order.  The exact table has
 * sum(ceil(len_i / chunk_size)) rows.  A caller that does not know the lengths on the
 * host (so never waits for the device) may pass any larger n_chunks, e.g. the bound
 * n_tokens / chunk_size + n_seqs: the rows after the last chunk are written as (-1, -1),
 * and moc_forward / moc_backward skip such rows.  A smaller n_chunks truncates the table.
 * Replaces the tensor arithmetic of prepare_chunk_indices, moc/ops.py:82-97. */
int moc_prepare_chunk_indices(const void* cu_seqlens, int32_t cu_seqlens_dtype, int64_t n_seqs,
                              int32_t chunk_size, int32_t* chunk_indices, int64_t n_chunks,
                              void* stream);

/* One module of a fused multi-module decode step (MoC modules sharing the routing
 * input z, as the q / k / v convolutions of an attention block do).  All pointers are
 * bf16 device memory: router weight [n_bases, z_dim]; basis [n_bases, kernel_size, dim];
 * x and out [batch, dim]; alpha [batch, n_bases] receives the router output; cache
 * [batch, dim, kernel_size] contiguous, updated in place as in moc_step. */
typedef struct moc_decode_module {
  int64_t dim;
  int32_t n_bases;            /* <= 16 */
  int32_t kernel_size;        /* 1..4 */
  int32_t activation;         /* 1 = fused SiLU */
  int32_t router_act;         /* 0 = softmax, 1 = exp */
  const void* weight;
  const void* basis;
  const void* x;
  void* cache;
  void* alpha;
  void* out;
} moc_decode_module;

#define MOC_DECODE_MAX_MODULES 4

/* Fused decode step of up to MOC_DECODE_MAX_MODULES modules that share z [batch, z_dim]:
 * one launch computes every module's router and, in the same clusters of CTAs, mixes
 * and convolves every module's channels and shifts its cache.  Results
 * agree with moc_router_forward followed by moc_step for each module within the bf16
 * tolerance: here the alpha.basis products enter an fp32 tensor-core sum exactly, where
 * moc_step (like the reference's decode kernel) rounds each product to bf16.  All modules share
 * one kernel_size; dim and z_dim must be multiples of 8 and every pointer 16-byte aligned.  Replaces, per module, the router
 * lines of MoC.forward (moc/api.py:383-388) and launch_update (moc/ops.py:341-362) with
 * one launch for all modules (the fused multi-module decode of the reference's
 * q / k / v usage, README.md:120-129). */
int moc_decode_step_multi(int32_t n_modules, const moc_decode_module* modules, int64_t batch,
                          int64_t z_dim, const void* z, void* stream);

/* Fused projection + convolution forward (bf16, fixed-length sequences):
 *
 *   out = MoC(h . weight^T)   h [batch * seq_len, in_dim], weight [dim, in_dim] (nn.Linear
 *                             layout), alpha [batch * seq_len, n_bases], basis [n_bases,
 *                             kernel_size, dim], out [batch * seq_len, dim]; all bf16,
 *                             row-major, contiguous, 16-byte aligned.
 *
 * The projection feeding a MoC module (the q, k or v slice of the reference's qkv_proj,
 * README.md:115-129) runs on the tensor cores (tcgen05, accumulators in tensor memory) with
 * the convolution as its epilogue: the projected x is rounded to bf16 on chip, as the
 * reference's bf16 qkv tensor is, and never written to memory (inference and prefill
 * without a cache; for training, moc_proj_forward_save below also writes it out).
 * Requires n_bases % 8 == 0 and n_bases <= 16, 1 <= kernel_size <= 8, in_dim % 8 == 0 and
 * dim % 8 == 0.  Not in the reference, which applies MoC after a separate projection GEMM. */
typedef struct moc_proj_problem {
  int64_t batch, seq_len;
  int64_t in_dim, dim;
  int32_t n_bases, kernel_size, activation;
  int32_t reserved;
  const void* h;
  const void* weight;
  const void* alpha;
  const void* basis;
  void* out;
} moc_proj_problem;
int moc_proj_forward(const moc_proj_problem* problem, void* stream);

/* The training form of moc_proj_forward: the same out, and x_out [batch * seq_len, dim] (bf16,
 * 16-byte aligned) receives the rounded projection x = h . weight^T that the convolution read.
 * The backward is then the convolution's (moc_backward on x, alpha, basis and dy gives dx,
 * dalpha, dbasis) followed by the projection's two GEMMs, dh = dx . weight and
 * dweight = dx^T . h, which are plain library GEMMs (the caller's BLAS).  Against the unfused
 * training forward (projection GEMM writing x, then moc_forward reading it back) this saves
 * one read of x and one launch.  x_out NULL is moc_proj_forward. */
int moc_proj_forward_save(const moc_proj_problem* problem, void* x_out, void* stream);

/* Several modules over one projection, in one launch: the reference's
 *   q, k, v = qkv_proj(x_norm).split(...);  q = q_conv(q, x_norm); ...
 * with weight = qkv_proj.weight [weight_rows, in_dim].  Module i takes weight rows
 * [row_offset, row_offset + dim) and writes out [batch * seq_len, dim] from its alpha
 * [batch * seq_len, n_bases] and basis [n_bases, kernel_size, dim].  h is read once for
 * all modules.  Every module has the same kernel_size; the requirements of
 * moc_proj_forward apply to each (n_bases % 8 == 0 and <= 16, dim % 8 == 0). */
#define MOC_PROJ_MAX_MODULES 4
typedef struct moc_proj_module {
  int64_t dim, row_offset;
  int32_t n_bases, activation;
  const void* alpha;
  const void* basis;
  void* out;
} moc_proj_module;
int moc_proj_forward_multi(int32_t n_modules, const moc_proj_module* modules, int64_t batch, int64_t seq_len,
                           int64_t in_dim, int32_t kernel_size, const void* h, const void* weight,
                           int64_t weight_rows, void* stream);

/* The training form of moc_proj_forward_multi: x_out holds n_modules pointers, module i's
 * rounded projection [batch * seq_len, dim_i] (bf16, 16-byte aligned; a NULL entry skips that
 * module's copy).  x_out NULL is moc_proj_forward_multi.  The backward as for
 * moc_proj_forward_save, with dweight's rows [row_offset, row_offset + dim) from module i. */
int moc_proj_forward_multi_save(int32_t n_modules, const moc_proj_module* modules, void* const* x_out,
                                int64_t batch, int64_t seq_len, int64_t in_dim, int32_t kernel_size, const void* h,
                                const void* weight, int64_t weight_rows, void* stream);

/* Gradient all-reduce over NVLink peer memory, for the data-parallel step (one process
 * per GPU).  The step's only collective sums the parameter gradients (conv_bases and
 * router) over ranks; at 640 KiB it is latency-bound, and this replaces the NCCL
 * all-reduce by one kernel that reads every rank's slice through CUDA IPC peer pointers.
 *
 * Setup, once per rank with its device current: moc_comm_create allocates this rank's
 * exchange buffer (2 x capacity fp32 plus flags; the only allocating calls of the
 * library are create / destroy) and writes its IPC handle (MOC_IPC_HANDLE_BYTES) to
 * handle_out; the caller gathers the world's handles in rank order (e.g. with
 * torch.distributed.all_gather_object) and passes them to moc_comm_connect.
 *
 * moc_comm_allreduce sums, in place on every rank, up to MOC_COMM_MAX_SEGMENTS device
 * arrays (data[i], counts[i] elements of dtypes[i]: fp32, fp16 or bf16), accumulating in
 * fp32 in rank order so every rank gets bitwise the same result.  Every rank must make
 * the same calls in the same order.  The call is stream-ordered and can be captured in a
 * CUDA graph.  A rank that waits too long for its peers (more than the poll limit) records
 * MOC_STATUS_WAIT_TIMEOUT in the communicator's status word (moc_comm_status) and in the
 * library's (moc_device_status), and leaves its data unchanged.  The ranks' call counters
 * then no longer pair up: before the next call, with no call in flight on any rank, every
 * rank calls moc_comm_reset and waits for it (and for the others, e.g. a host barrier).
 * No counterpart in the reference, which trains in one process. */
#define MOC_COMM_MAX_RANKS 8
#define MOC_COMM_MAX_SEGMENTS 4
#define MOC_IPC_HANDLE_BYTES 64
typedef struct moc_comm moc_comm;
int moc_comm_create(int32_t rank, int32_t world, int64_t capacity, moc_comm** comm, void* handle_out);
int moc_comm_connect(moc_comm* comm, const void* handles);
int moc_comm_allreduce(moc_comm* comm, int32_t n_segments, void* const* data, const int64_t* counts,
                       const int32_t* dtypes, void* stream);
int moc_comm_destroy(moc_comm* comm);
/* Polls of a peer's flag before a call gives up (0 restores the default, 2^22). */
int moc_comm_set_poll_limit(moc_comm* comm, uint32_t poll_limit);
/* This communicator's status word: MOC_STATUS_* bits of its calls since the last clear
 * (synchronous: reads device memory). */
int moc_comm_status(moc_comm* comm, int* status, int clear);
/* Zeroes this rank's flags, call counters and status word (stream-ordered): the recovery
 * after a timeout, described above. */
int moc_comm_reset(moc_comm* comm, void* stream);
/* Diagnostic: runs the all-reduce kernel as rank 0 of a world of two whose rank 1 never
 * calls (on a fixed array of the library), so every wait gives up after poll_limit polls
 * and records MOC_STATUS_WAIT_TIMEOUT (moc_device_status).  Used by the tests of the
 * bounded-wait path. */
int moc_comm_wait_timeout_probe(uint32_t poll_limit, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOC_B200_H */
