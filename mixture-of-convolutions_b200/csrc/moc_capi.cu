// extern "C" entry points declared in include/moc_b200.h: argument checks, then
// dispatch to the tensor-core kernels (bf16 shapes they support) or the generic
// CUDA-core kernels.  No entry point allocates memory or synchronises the host.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_tma.cuh"

namespace moc {

static thread_local std::string g_last_cuda_error;
static int g_kernel_path = 0;  // 0 = auto, 1 = generic CUDA-core kernels only
static std::atomic<uint64_t> g_launches{0};

void note_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

int note_cuda(cudaError_t e) {
  if (e == cudaSuccess) return MOC_OK;
  g_last_cuda_error = std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
  return MOC_ERR_CUDA;
}

static bool valid_float_dtype(int d) { return d == MOC_DTYPE_F32 || d == MOC_DTYPE_F16 || d == MOC_DTYPE_BF16; }
static bool valid_index_dtype(int d) { return d == MOC_INDEX_I32 || d == MOC_INDEX_I64; }

static int check_problem(const moc_problem* p) {
  if (p == nullptr) return MOC_ERR_INVALID_ARGUMENT;
  if (p->x_dtype != MOC_DTYPE_F32 && p->x_dtype != MOC_DTYPE_BF16) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (!valid_float_dtype(p->alpha_dtype) || !valid_float_dtype(p->basis_dtype)) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (p->dim <= 0 || p->n_bases <= 0 || p->kernel_size <= 0 || p->n_tokens < 0) return MOC_ERR_INVALID_ARGUMENT;
  if (p->n_bases > kMaxBasesSimt || p->kernel_size > kMaxKernelSize) return MOC_ERR_UNSUPPORTED_SHAPE;
  if (p->activation != 0 && p->activation != 1) return MOC_ERR_INVALID_ARGUMENT;
  if (p->cu_seqlens == nullptr) {
    if (p->batch <= 0 || p->seq_len <= 0 || p->batch * p->seq_len != p->n_tokens) return MOC_ERR_INVALID_ARGUMENT;
  } else {
    if (p->n_seqs < 1 || p->chunk_size <= 0 || p->n_chunks < 0) return MOC_ERR_INVALID_ARGUMENT;
    if (!valid_index_dtype(p->cu_seqlens_dtype) || !valid_index_dtype(p->chunk_indices_dtype))
      return MOC_ERR_UNSUPPORTED_DTYPE;
    if (p->n_chunks > 0 && p->chunk_indices == nullptr) return MOC_ERR_INVALID_ARGUMENT;
  }
  if (p->halo != nullptr) {  // a cache precedes fixed-length sequences only
    if (p->cu_seqlens != nullptr) return MOC_ERR_INVALID_ARGUMENT;
    if (p->halo_strides[0] < 0 || p->halo_strides[1] < 0 || p->halo_strides[2] < 0) return MOC_ERR_INVALID_ARGUMENT;
  }
  return MOC_OK;
}

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                      uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (encode == nullptr) {
    g_last_cuda_error = "cuTensorMapEncodeTiled entry point unavailable";
    return MOC_ERR_CUDA;
  }
  // The encoding is a driver call and needs a current context on this thread.  A thread
  // that has made no runtime call of this library yet (the autograd engine's device
  // thread, say) may have none: bind the device's primary context once per thread.
  thread_local uint64_t bound = 0;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce == cudaSuccess && dev >= 0 && dev < 64 && !((bound >> dev) & 1)) {
    ce = cudaSetDevice(dev);
    if (ce == cudaSuccess) bound |= uint64_t{1} << dev;
  }
  if (ce != cudaSuccess) return note_cuda(ce);
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                            CU_TENSOR_MAP_INTERLEAVE_NONE,
                            swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                            : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                            : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return MOC_ERR_CUDA;
  }
  return MOC_OK;
}

static bool use_tc(const moc_problem& p) { return g_kernel_path != MOC_PATH_GENERIC && tc_conv_supported(p); }

}  // namespace moc

using namespace moc;

extern "C" {

const char* moc_version(void) { return "moc_b200 0.1.0 sm_100a"; }

const char* moc_error_string(int code) {
  switch (code) {
    case MOC_OK: return "ok";
    case MOC_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MOC_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case MOC_ERR_UNSUPPORTED_SHAPE: return "unsupported shape (n_bases > 128 or kernel_size > 64)";
    case MOC_ERR_MISALIGNED: return "pointer not aligned for vector access";
    case MOC_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case MOC_ERR_CUDA: return "CUDA error (see moc_last_cuda_error)";
    case MOC_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the fixed MOC_NOALLOC_SCRATCH_BYTES array (use the workspace entry point)";
    default: return "unknown error code";
  }
}

const char* moc_last_cuda_error(void) { return g_last_cuda_error.c_str(); }

uint64_t moc_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int moc_device_status(int* status, int clear) {
  if (status == nullptr) return MOC_ERR_INVALID_ARGUMENT;
  int r = 0, c = 0, m = 0, j = 0, d = 0;
  int rc = router_status(&r, clear != 0);
  if (rc == MOC_OK) rc = conv_status(&c, clear != 0);
  int c5 = 0;
  if (rc == MOC_OK) rc = bwd5_status(&c5, clear != 0);
  c |= c5;
  if (rc == MOC_OK) rc = comm_status(&m, clear != 0);
  if (rc == MOC_OK) rc = proj_status(&j, clear != 0);
  if (rc == MOC_OK) rc = decode_status(&d, clear != 0);
  if (rc != MOC_OK) return rc;
  *status = r | c | m | j | d;
  return MOC_OK;
}

int moc_wait_timeout_probe(uint32_t poll_limit, void* stream) {
  return wait_timeout_probe(poll_limit, static_cast<cudaStream_t>(stream));
}

int moc_cluster_wait_timeout_probe(uint32_t poll_limit, void* stream) {
  return decode_wait_timeout_probe(poll_limit, static_cast<cudaStream_t>(stream));
}

// Selects the kernel family: automatic (tensor cores where supported), generic CUDA-core
// kernels for every shape, or automatic with the warp-level conv backward for every shape.
// All compute the full result.
int moc_set_kernel_path(int path) {
  if (path != MOC_PATH_AUTO && path != MOC_PATH_GENERIC && path != MOC_PATH_WARP_BACKWARD)
    return MOC_ERR_INVALID_ARGUMENT;
  g_kernel_path = path;
  tc_allow_bwd5(path == MOC_PATH_AUTO);
  return MOC_OK;
}

int moc_forward(const moc_problem* p, const void* x, const void* alpha, const void* basis, void* out,
                void* stream) {
  int rc = check_problem(p);
  if (rc != MOC_OK) return rc;
  if (p->n_tokens == 0) return MOC_OK;
  if (!x || !alpha || !basis || !out) return MOC_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_tc(*p)) return tc_forward(*p, x, alpha, basis, out, st);
  return simt_forward(*p, x, alpha, basis, out, st);
}

size_t moc_backward_workspace_bytes(const moc_problem* p) {
  if (check_problem(p) != MOC_OK) return 0;
  return use_tc(*p) ? tc_backward_ws(*p) : simt_backward_ws(*p);
}

int moc_backward(const moc_problem* p, const void* x, const void* alpha, const void* basis, const void* dy,
                 void* dx, void* dalpha, void* dbasis, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_problem(p);
  if (rc != MOC_OK) return rc;
  if (!basis || !dbasis) return MOC_ERR_INVALID_ARGUMENT;
  if (p->n_tokens > 0 && (!x || !alpha || !dy || !dalpha)) return MOC_ERR_INVALID_ARGUMENT;
  // the tensor-core backward writes its dalpha partials 16 bytes at a time
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return MOC_ERR_MISALIGNED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_tc(*p)) {
    if (workspace_bytes < tc_backward_ws(*p)) return MOC_ERR_WORKSPACE_TOO_SMALL;
    return tc_backward(*p, x, alpha, basis, dy, dx, dalpha, dbasis, workspace, workspace_bytes, st);
  }
  if (workspace_bytes < simt_backward_ws(*p)) return MOC_ERR_WORKSPACE_TOO_SMALL;
  return simt_backward(*p, x, alpha, basis, dy, dx, dalpha, dbasis, workspace, workspace_bytes, st);
}

int moc_step(int64_t batch, int64_t dim, int32_t n_bases, int32_t kernel_size, int32_t x_dtype,
             int32_t alpha_dtype, int32_t basis_dtype, int32_t activation, const void* x, const void* alpha,
             const void* basis, void* cache, const int64_t cache_strides[3], void* out, void* stream) {
  if (x_dtype != MOC_DTYPE_F32 && x_dtype != MOC_DTYPE_BF16) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (!valid_float_dtype(alpha_dtype) || !valid_float_dtype(basis_dtype)) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || dim <= 0 || n_bases <= 0 || kernel_size <= 0) return MOC_ERR_INVALID_ARGUMENT;
  if (activation != 0 && activation != 1) return MOC_ERR_INVALID_ARGUMENT;
  if (batch > 65535) return MOC_ERR_UNSUPPORTED_SHAPE;
  if (batch == 0) return MOC_OK;
  if (!x || !alpha || !basis || !cache || !cache_strides || !out) return MOC_ERR_INVALID_ARGUMENT;
  return simt_step(batch, dim, n_bases, kernel_size, x_dtype, alpha_dtype, basis_dtype, activation, x, alpha,
                   basis, cache, cache_strides, out, static_cast<cudaStream_t>(stream));
}

int moc_decode_step_multi(int32_t n_modules, const moc_decode_module* modules, int64_t batch, int64_t z_dim,
                          const void* z, void* stream) {
  if (n_modules < 1 || n_modules > MOC_DECODE_MAX_MODULES || !modules) return MOC_ERR_INVALID_ARGUMENT;
  if (batch < 0 || z_dim <= 0) return MOC_ERR_INVALID_ARGUMENT;
  if (z_dim % 8 != 0 || batch > (int64_t{1} << 30) || z_dim > (int64_t{1} << 40)) return MOC_ERR_UNSUPPORTED_SHAPE;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int32_t S = modules[0].kernel_size;
  int64_t blocks = 0;
  for (int i = 0; i < n_modules; ++i) {
    const moc_decode_module& m = modules[i];
    if (m.dim <= 0 || m.n_bases <= 0 || m.kernel_size <= 0) return MOC_ERR_INVALID_ARGUMENT;
    if ((m.activation != 0 && m.activation != 1) || (m.router_act != 0 && m.router_act != 1))
      return MOC_ERR_INVALID_ARGUMENT;
    if (m.n_bases > 16 || m.kernel_size > 4 || m.kernel_size != S || m.dim % 8 != 0 || m.dim > (int64_t{1} << 40))
      return MOC_ERR_UNSUPPORTED_SHAPE;
    if (!m.weight || !m.basis || !m.x || !m.cache || !m.alpha || !m.out) return MOC_ERR_INVALID_ARGUMENT;
    if (!a16(m.weight) || !a16(m.basis) || !a16(m.x) || !a16(m.cache) || !a16(m.alpha) || !a16(m.out))
      return MOC_ERR_MISALIGNED;
    blocks += (m.dim + 127) / 128;
  }
  if (blocks > (int64_t{1} << 30)) return MOC_ERR_UNSUPPORTED_SHAPE;
  if (batch == 0) return MOC_OK;
  if (!z) return MOC_ERR_INVALID_ARGUMENT;
  if (!a16(z)) return MOC_ERR_MISALIGNED;
  return decode_step_multi(n_modules, modules, batch, z_dim, z, static_cast<cudaStream_t>(stream));
}

int moc_proj_forward_multi(int32_t n_modules, const moc_proj_module* modules, int64_t batch, int64_t seq_len,
                           int64_t in_dim, int32_t kernel_size, const void* h, const void* weight,
                           int64_t weight_rows, void* stream) {
  return moc_proj_forward_multi_save(n_modules, modules, nullptr, batch, seq_len, in_dim, kernel_size, h, weight,
                                     weight_rows, stream);
}

int moc_proj_forward_multi_save(int32_t n_modules, const moc_proj_module* modules, void* const* x_out,
                                int64_t batch, int64_t seq_len, int64_t in_dim, int32_t kernel_size, const void* h,
                                const void* weight, int64_t weight_rows, void* stream) {
  if (n_modules < 1 || n_modules > MOC_PROJ_MAX_MODULES || !modules) return MOC_ERR_INVALID_ARGUMENT;
  if (batch < 0 || seq_len < 0 || in_dim <= 0 || kernel_size <= 0 || weight_rows <= 0) return MOC_ERR_INVALID_ARGUMENT;
  if (kernel_size > 8 || in_dim % 8 != 0) return MOC_ERR_UNSUPPORTED_SHAPE;
  // tensor-map coordinates are 32-bit
  const int64_t lim = (int64_t{1} << 31) - 1024;
  if (seq_len > lim || (seq_len > 0 && batch > lim / seq_len) || in_dim > lim || weight_rows > lim)
    return MOC_ERR_UNSUPPORTED_SHAPE;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  for (int i = 0; i < n_modules; ++i) {
    const moc_proj_module& m = modules[i];
    if (m.dim <= 0 || m.n_bases <= 0 || m.row_offset < 0) return MOC_ERR_INVALID_ARGUMENT;
    if (m.activation != 0 && m.activation != 1) return MOC_ERR_INVALID_ARGUMENT;
    if (m.row_offset > weight_rows - m.dim) return MOC_ERR_INVALID_ARGUMENT;  // rows past the weight
    if (m.n_bases % 8 != 0 || m.n_bases > 16 || m.dim % 8 != 0) return MOC_ERR_UNSUPPORTED_SHAPE;
    if (batch > 0 && seq_len > 0) {
      if (!m.alpha || !m.basis || !m.out) return MOC_ERR_INVALID_ARGUMENT;
      if (!a16(m.alpha) || !a16(m.basis) || !a16(m.out)) return MOC_ERR_MISALIGNED;
      if (x_out && !a16(x_out[i])) return MOC_ERR_MISALIGNED;  // NULL (no copy) is aligned
    }
  }
  if (batch == 0 || seq_len == 0) return MOC_OK;
  if (!h || !weight) return MOC_ERR_INVALID_ARGUMENT;
  if (!a16(h) || !a16(weight)) return MOC_ERR_MISALIGNED;
  return proj_forward_multi(n_modules, modules, x_out, batch, seq_len, in_dim, kernel_size, h, weight, weight_rows,
                            static_cast<cudaStream_t>(stream));
}

int moc_proj_forward(const moc_proj_problem* p, void* stream) { return moc_proj_forward_save(p, nullptr, stream); }

int moc_proj_forward_save(const moc_proj_problem* p, void* x_out, void* stream) {
  if (!p) return MOC_ERR_INVALID_ARGUMENT;
  if (p->dim <= 0) return MOC_ERR_INVALID_ARGUMENT;
  if (p->dim % 8 != 0) return MOC_ERR_UNSUPPORTED_SHAPE;
  moc_proj_module m{};
  m.dim = p->dim;
  m.row_offset = 0;
  m.n_bases = p->n_bases;
  m.activation = p->activation;
  m.alpha = p->alpha;
  m.basis = p->basis;
  m.out = p->out;
  void* const xs[1] = {x_out};
  return moc_proj_forward_multi_save(1, &m, xs, p->batch, p->seq_len, p->in_dim, p->kernel_size, p->h, p->weight,
                                     p->dim, stream);
}

int moc_comm_create(int32_t rank, int32_t world, int64_t capacity, moc_comm** comm, void* handle_out) {
  if (!comm || !handle_out || world < 1 || world > MOC_COMM_MAX_RANKS || rank < 0 || rank >= world || capacity <= 0)
    return MOC_ERR_INVALID_ARGUMENT;
  if (capacity > (int64_t{1} << 34)) return MOC_ERR_UNSUPPORTED_SHAPE;
  CommImpl* c = nullptr;
  const int rc = comm_create(rank, world, capacity, &c, handle_out);
  if (rc == MOC_OK) *comm = reinterpret_cast<moc_comm*>(c);
  return rc;
}

int moc_comm_connect(moc_comm* comm, const void* handles) {
  if (!comm || !handles) return MOC_ERR_INVALID_ARGUMENT;
  return comm_connect(reinterpret_cast<CommImpl*>(comm), handles);
}

int moc_comm_allreduce(moc_comm* comm, int32_t n_segments, void* const* data, const int64_t* counts,
                       const int32_t* dtypes, void* stream) {
  if (!comm || n_segments < 0 || n_segments > MOC_COMM_MAX_SEGMENTS || (n_segments > 0 && (!data || !counts || !dtypes)))
    return MOC_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < n_segments; ++i) {
    if (!valid_float_dtype(dtypes[i])) return MOC_ERR_UNSUPPORTED_DTYPE;
    if (counts[i] < 0 || (counts[i] > 0 && !data[i])) return MOC_ERR_INVALID_ARGUMENT;
  }
  return comm_allreduce(reinterpret_cast<CommImpl*>(comm), n_segments, data, counts, dtypes,
                        static_cast<cudaStream_t>(stream));
}

int moc_comm_set_poll_limit(moc_comm* comm, uint32_t poll_limit) {
  if (!comm) return MOC_ERR_INVALID_ARGUMENT;
  comm_set_poll_limit(reinterpret_cast<CommImpl*>(comm), poll_limit);
  return MOC_OK;
}

int moc_comm_status(moc_comm* comm, int* status, int clear) {
  if (!comm || !status) return MOC_ERR_INVALID_ARGUMENT;
  return comm_own_status(reinterpret_cast<CommImpl*>(comm), status, clear != 0);
}

int moc_comm_reset(moc_comm* comm, void* stream) {
  if (!comm) return MOC_ERR_INVALID_ARGUMENT;
  return comm_reset(reinterpret_cast<CommImpl*>(comm), static_cast<cudaStream_t>(stream));
}

int moc_comm_wait_timeout_probe(uint32_t poll_limit, void* stream) {
  return comm_wait_timeout_probe(poll_limit, static_cast<cudaStream_t>(stream));
}

int moc_comm_destroy(moc_comm* comm) {
  if (!comm) return MOC_ERR_INVALID_ARGUMENT;
  return comm_destroy(reinterpret_cast<CommImpl*>(comm));
}

int moc_router_forward(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype, int32_t router_act,
                       const void* z, const void* weight, void* alpha, void* stream) {
  if (!valid_float_dtype(dtype)) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (n_tokens < 0 || z_dim <= 0 || n_bases <= 0 || (router_act != 0 && router_act != 1))
    return MOC_ERR_INVALID_ARGUMENT;
  if (n_bases > kMaxBasesSimt) return MOC_ERR_UNSUPPORTED_SHAPE;
  if (n_tokens == 0) return MOC_OK;
  if (!z || !weight || !alpha) return MOC_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (g_kernel_path != MOC_PATH_GENERIC && tc_router_supported(n_tokens, z_dim, n_bases, dtype))
    return tc_router_forward(n_tokens, z_dim, n_bases, router_act, z, weight, alpha, st);
  return simt_router_forward(n_tokens, z_dim, n_bases, dtype, router_act, z, weight, alpha, st);
}

size_t moc_router_backward_workspace_bytes(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype) {
  if (n_tokens < 0 || z_dim <= 0 || n_bases <= 0) return 0;
  if (g_kernel_path != MOC_PATH_GENERIC && tc_router_supported(n_tokens, z_dim, n_bases, dtype))
    return tc_router_backward_ws(n_tokens, z_dim, n_bases);
  return simt_router_backward_ws(n_tokens, z_dim, n_bases);
}

int moc_router_backward(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype, int32_t router_act,
                        const void* z, const void* weight, const void* alpha, const void* dalpha,
                        int32_t dalpha_dtype, void* dz, void* dweight, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!valid_float_dtype(dtype) || !valid_float_dtype(dalpha_dtype)) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (n_tokens < 0 || z_dim <= 0 || n_bases <= 0 || (router_act != 0 && router_act != 1))
    return MOC_ERR_INVALID_ARGUMENT;
  if (n_bases > kMaxBasesSimt) return MOC_ERR_UNSUPPORTED_SHAPE;
  if (n_tokens > 0 && (!z || !weight || !alpha || !dalpha)) return MOC_ERR_INVALID_ARGUMENT;
  // the workspace holds fp32 partials; 16-byte alignment, as for moc_backward's
  if (dweight != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return MOC_ERR_MISALIGNED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (g_kernel_path != MOC_PATH_GENERIC && tc_router_supported(n_tokens, z_dim, n_bases, dtype)) {
    if (workspace_bytes < tc_router_backward_ws(n_tokens, z_dim, n_bases)) return MOC_ERR_WORKSPACE_TOO_SMALL;
    return tc_router_backward(n_tokens, z_dim, n_bases, router_act, z, weight, alpha, dalpha, dalpha_dtype, dz,
                              dweight, workspace, workspace_bytes, st);
  }
  if (workspace_bytes < simt_router_backward_ws(n_tokens, z_dim, n_bases)) return MOC_ERR_WORKSPACE_TOO_SMALL;
  return simt_router_backward(n_tokens, z_dim, n_bases, dtype, router_act, z, weight, alpha, dalpha, dalpha_dtype,
                              dz, dweight, workspace, workspace_bytes, st);
}

int moc_router_backward_noalloc(int64_t n_tokens, int64_t z_dim, int32_t n_bases, int32_t dtype, int32_t router_act,
                                const void* z, const void* weight, const void* alpha, const void* dalpha,
                                int32_t dalpha_dtype, void* dz, void* dweight, void* stream) {
  if (!valid_float_dtype(dtype) || !valid_float_dtype(dalpha_dtype)) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (n_tokens < 0 || z_dim <= 0 || n_bases <= 0 || (router_act != 0 && router_act != 1))
    return MOC_ERR_INVALID_ARGUMENT;
  if (dtype != MOC_DTYPE_BF16) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (n_tokens == 0) return MOC_OK;
  if (!tc_router_supported(n_tokens, z_dim, n_bases, dtype)) return MOC_ERR_UNSUPPORTED_SHAPE;
  if (!z || !weight || !alpha || !dalpha) return MOC_ERR_INVALID_ARGUMENT;
  return tc_router_backward_noalloc(n_tokens, z_dim, n_bases, router_act, z, weight, alpha, dalpha, dalpha_dtype, dz,
                                    dweight, static_cast<cudaStream_t>(stream));
}

int moc_prepare_chunk_indices(const void* cu_seqlens, int32_t cu_seqlens_dtype, int64_t n_seqs, int32_t chunk_size,
                              int32_t* chunk_indices, int64_t n_chunks, void* stream) {
  if (!valid_index_dtype(cu_seqlens_dtype)) return MOC_ERR_UNSUPPORTED_DTYPE;
  if (n_seqs < 0 || chunk_size <= 0 || n_chunks < 0) return MOC_ERR_INVALID_ARGUMENT;
  if (n_chunks > 0 && (!cu_seqlens || !chunk_indices)) return MOC_ERR_INVALID_ARGUMENT;
  return build_chunk_indices(cu_seqlens, cu_seqlens_dtype == MOC_INDEX_I64, n_seqs, chunk_size, chunk_indices,
                             n_chunks, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
