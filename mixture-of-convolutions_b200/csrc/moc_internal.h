// Internal launcher interface between the C ABI (moc_capi.cu) and the kernel files.
// Launchers validate nothing the C ABI already checked; they return MOC_* codes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/moc_b200.h"

namespace moc {

// ---- generic CUDA-core path: any dtype mix, any K <= 128, any S <= 64 (moc_simt.cu)
int simt_forward(const moc_problem& p, const void* x, const void* alpha, const void* basis, void* out,
                 cudaStream_t st);
size_t simt_backward_ws(const moc_problem& p);
int simt_backward(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy,
                  void* dx, void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st);
int simt_step(int64_t B, int64_t D, int K, int S, int x_dtype, int a_dtype, int b_dtype, int act, const void* x,
              const void* alpha, const void* basis, void* cache, const int64_t cs[3], void* out,
              cudaStream_t st);
int simt_router_forward(int64_t N, int64_t Dz, int K, int dtype, int act, const void* z, const void* w,
                        void* alpha, cudaStream_t st);
size_t simt_router_backward_ws(int64_t N, int64_t Dz, int K);
int simt_router_backward(int64_t N, int64_t Dz, int K, int dtype, int act, const void* z, const void* w,
                         const void* alpha, const void* dalpha, int da_dtype, void* dz, void* dw, void* ws,
                         size_t ws_bytes, cudaStream_t st);
int build_chunk_indices(const void* cu, int cu_i64, int64_t n_seqs, int chunk, int32_t* out, int64_t n_chunks,
                        cudaStream_t st);

// ---- tensor-core path for bf16 x/alpha/basis (moc_tc.cu); *_supported says whether
// the problem fits its templates, otherwise the caller uses the generic path.
bool tc_conv_supported(const moc_problem& p);
int tc_forward(const moc_problem& p, const void* x, const void* alpha, const void* basis, void* out,
               cudaStream_t st);
size_t tc_backward_ws(const moc_problem& p);
int tc_backward(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy,
                void* dx, void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st);

// fixed-order sum of the conv backward's per-CTA partials into dalpha / dbasis (moc_tc.cu)
int tc_finalize(const float* da_part, int64_t n_slices, int64_t nk, void* dalpha, int adt, const float* db_part,
                int64_t groups, int64_t ksd, void* dbasis, int bdt, cudaStream_t st);
// lets tc_backward use the tcgen05 backward for the shapes it serves (default) or not
void tc_allow_bwd5(bool allowed);

// ---- conv backward with the dalpha / dbasis contractions on tcgen05 (moc_bwd5.cu), for the
// bf16 shapes whose dbasis accumulators do not fit the warp-level kernel's registers
// (17..32 bases, 5..8 taps)
bool tc5_supported(const moc_problem& p);
size_t tc5_backward_ws(const moc_problem& p);
int tc5_backward(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy, void* dx,
                 void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st);
int bwd5_status(int* out, bool clear);

// ---- tensor-core router for bf16 (moc_router_tc.cu)
bool tc_router_supported(int64_t N, int64_t Dz, int K, int dtype);
int tc_router_forward(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, void* alpha,
                      cudaStream_t st);
size_t tc_router_backward_ws(int64_t N, int64_t Dz, int K);
int tc_router_backward(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, const void* alpha,
                       const void* dalpha, int da_dtype, void* dz, void* dw, void* ws, size_t ws_bytes,
                       cudaStream_t st);

// router backward with its scratch in a fixed device array (moc_router_tc.cu)
int tc_router_backward_noalloc(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, const void* alpha,
                               const void* dalpha, int da_dtype, void* dz, void* dw, cudaStream_t st);

// fused decode step of up to MOC_DECODE_MAX_MODULES modules sharing z (moc_decode.cu)
int decode_step_multi(int n, const moc_decode_module* mods, int64_t B, int64_t Dz, const void* z, cudaStream_t st);

// fused projection GEMM (tcgen05) + convolution forward (moc_proj.cu); x_out (NULL, or one
// pointer per module, each NULL or [batch * seq_len, dim]) receives the rounded projection
int proj_forward_multi(int n, const moc_proj_module* mods, void* const* x_out, int64_t batch, int64_t seq_len,
                       int64_t in_dim, int S, const void* h, const void* weight, int64_t weight_rows, cudaStream_t st);
int proj_status(int* out, bool clear);

// gradient all-reduce over NVLink peer memory (moc_comm.cu); CommImpl is the object
// behind the C ABI's opaque moc_comm
struct CommImpl;
int comm_create(int rank, int world, int64_t capacity, CommImpl** out, void* handle_out);
int comm_connect(CommImpl* c, const void* handles);
int comm_allreduce(CommImpl* c, int n_seg, void* const* data, const int64_t* n, const int32_t* dtype,
                   cudaStream_t st);
int comm_destroy(CommImpl* c);
int comm_status(int* out, bool clear);
void comm_set_poll_limit(CommImpl* c, uint32_t limit);
int comm_reset(CommImpl* c, cudaStream_t st);
int comm_own_status(CommImpl* c, int* out, bool clear);
int comm_wait_timeout_probe(uint32_t limit, cudaStream_t st);

// device status words of the TMA-staged kernels (bounded-wait timeouts), read/cleared
// by moc_device_status(); and a probe kernel that exercises the timeout path.
int router_status(int* out, bool clear);
int conv_status(int* out, bool clear);
int decode_status(int* out, bool clear);
int decode_wait_timeout_probe(uint32_t limit, cudaStream_t st);
int wait_timeout_probe(uint32_t limit, cudaStream_t st);

constexpr int kMaxBasesSimt = 128;
constexpr int kMaxKernelSize = 64;

}  // namespace moc
