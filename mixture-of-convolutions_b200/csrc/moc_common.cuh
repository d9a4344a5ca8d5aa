// Shared device helpers for the MoC kernels: dtype conversion, the bf16 rounding
// points of the reference's bf16 compute mode, and the token-row mapping that turns
// a fixed-length batch or a packed varlen chunk list into row ranges.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/moc_b200.h"

namespace moc {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- programmatic dependent launch
//
// The kernels of a training step are launched as programmatic dependents of the kernel
// before them on the stream (launch_pdl): a kernel may start while its predecessor
// finishes, runs its set-up (shared memory, barriers, tensor-map prefetch, loads of the
// basis / router weight, which no kernel of the chain writes) and then waits in
// griddep_wait() for the predecessor grid to complete, with its writes visible.  Every
// read of an activation, gradient or partial sum, and every global write, comes after that
// wait, so no kernel touches memory a running predecessor may still use (including memory
// the caching allocator handed out again).  Each kernel lets its own dependent start at
// once (griddep_launch_dependents); the dependent still waits for it to complete.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- conversions

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f32<bf16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Load element `i` of a tensor whose storage type is only known at run time.
// The branch is uniform across a warp, so it costs a predicate, not divergence.
__device__ __forceinline__ float ld_any(const void* p, int dtype, int64_t i) {
  if (dtype == MOC_DTYPE_BF16) return __bfloat162float(static_cast<const bf16*>(p)[i]);
  if (dtype == MOC_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void st_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == MOC_DTYPE_BF16)
    static_cast<bf16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == MOC_DTYPE_F16)
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    static_cast<float*>(p)[i] = v;
}

// In bf16 compute mode the reference rounds alpha, basis and the dz*x product to
// bf16 before each contraction (moc/kernels.py:92-95, 125-128, 390-392); in fp32
// mode values pass through unchanged.
template <bool BF16>
__device__ __forceinline__ float cround(float v) {
  if constexpr (BF16) {
    return __bfloat162float(__float2bfloat16_rn(v));
  } else {
    return v;
  }
}

__device__ __forceinline__ int64_t ld_index(const void* p, int is_i64, int64_t i) {
  return is_i64 ? static_cast<const int64_t*>(p)[i] : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// SiLU and its derivative, in the reference's form (moc/kernels.py:132-133, 231-232).
__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float dsilu_f(float v) {
  const float sig = 1.0f / (1.0f + expf(-v));
  return sig * (1.0f + v * (1.0f - sig));
}

// Logistic sigmoid for the kernels whose outputs are bf16: 0.5 + 0.5 tanh(v / 2) with one
// tanh.approx.f32 (maximum relative error about 2^-11, under the 2^-9 rounding step of a
// bf16 result) in place of an exponential and an IEEE division.
__device__ __forceinline__ float sigmoid_bf(float v) {
  float t;
  asm("tanh.approx.f32 %0, %1;\n" : "=f"(t) : "f"(0.5f * v));
  return fmaf(0.5f, t, 0.5f);
}
__device__ __forceinline__ float silu_bf(float v) { return v * sigmoid_bf(v); }
__device__ __forceinline__ float dsilu_bf(float v) {
  const float sig = sigmoid_bf(v);
  return sig * fmaf(v, 1.0f - sig, 1.0f);
}

// The same for a pair of values with packed fp32x2 arithmetic: with h = v / 2,
// silu(v) = h + h tanh(h), and sigmoid(v) = 1/2 + tanh(h) / 2.
__device__ __forceinline__ float2 tanh2_approx(float2 h) {
  float2 t;
  asm("tanh.approx.f32 %0, %1;\n" : "=f"(t.x) : "f"(h.x));
  asm("tanh.approx.f32 %0, %1;\n" : "=f"(t.y) : "f"(h.y));
  return t;
}
__device__ __forceinline__ float2 silu_bf2(float v0, float v1) {
  const float2 h = __fmul2_rn(make_float2(v0, v1), make_float2(0.5f, 0.5f));
  return __ffma2_rn(h, tanh2_approx(h), h);
}
// dsilu(v) = sig (1 + v (1 - sig))
__device__ __forceinline__ float2 dsilu_bf2(float v0, float v1) {
  const float2 v = make_float2(v0, v1), half = make_float2(0.5f, 0.5f);
  const float2 t = tanh2_approx(__fmul2_rn(v, half));
  const float2 sig = __ffma2_rn(t, half, half);
  const float2 one_m = __ffma2_rn(t, make_float2(-0.5f, -0.5f), half);
  return __fmul2_rn(sig, __ffma2_rn(v, one_m, make_float2(1.f, 1.f)));
}

// ------------------------------------------------------------------ partial sums

// Fixed-order sum of the `parts` partial rows (row p at base + p * stride) at element i, by the
// four lanes sub = 0..3 of a lane quad (lanes 4m .. 4m + 3, all with the same i): lane sub adds
// rows sub, sub + 4, ... in order, then the quad's four sums meet in a fixed shuffle tree, so
// every call gives the same bits.  The shuffles name only the quad, so quads of one warp may
// take different branches.  For short sums over many parts: four loads in flight per element.
__device__ __forceinline__ float quad_part_sum(const float* __restrict__ base, int64_t parts, int64_t stride,
                                               int64_t i, int sub) {
  const unsigned quad = 0xfu << (threadIdx.x & 28);
  float s = 0.f;
#pragma unroll 4
  for (int64_t p = sub; p < parts; p += 4) s += __ldg(base + p * stride + i);
  s += __shfl_xor_sync(quad, s, 1);
  s += __shfl_xor_sync(quad, s, 2);
  return s;
}

// ------------------------------------------------------------------ row mapping

// A work item is a run of consecutive token rows [r0, r1) inside one sequence whose
// rows are [seq_start, seq_end).  Fixed length: item i is tile (i % tiles) of sequence
// (i / tiles).  Varlen: item i is chunk_indices[i] = (seq_id, chunk) of chunk_size rows,
// the reference's packed-chunk scheme (moc/kernels.py:57-76).  Items whose indices point
// outside the problem are reported empty rather than read out of bounds.
struct RowMap {
  int64_t batch = 0, seq_len = 0, n_tokens = 0;
  int64_t tiles_per_seq = 0;
  int32_t tile = 0;
  int32_t idx32 = 0;  // fixed length with fewer than 2^31 items: item() divides in 32 bits
  int32_t varlen = 0;
  const void* cu = nullptr;
  int32_t cu_i64 = 0;
  int64_t n_seqs = 0;
  const void* chunks = nullptr;
  int32_t ch_i64 = 0;
  int64_t n_chunks = 0;
  int32_t chunk_size = 0;

  // fixed length with a cache: the tokens before each sequence (cache [batch, D, S], slot S-1
  // newest), read by the causal taps instead of zeros
  const void* halo = nullptr;
  int64_t hs0 = 0, hs1 = 0, hs2 = 0;
  int32_t halo_S = 0, halo_dt = 0;

  __host__ __device__ int64_t n_items() const { return varlen ? n_chunks : batch * tiles_per_seq; }

  // x value of token `src` < `seq_start` (m = seq_start - src tokens back) for channel d:
  // the cache slot S - m when a cache is attached and m < S, else 0
  __device__ __forceinline__ float halo_at(int64_t seq_start, int64_t src, int64_t d) const {
    if (halo == nullptr || varlen) return 0.f;
    const int64_t m = seq_start - src;
    if (m < 1 || m >= halo_S) return 0.f;
    const int64_t b = seq_start / seq_len;
    return ld_any(halo, halo_dt, b * hs0 + d * hs1 + (halo_S - m) * hs2);
  }
  // Rows per item (upper bound).
  __host__ __device__ int32_t item_rows() const { return varlen ? chunk_size : tile; }

  __device__ __forceinline__ bool item(int64_t i, int64_t& seq_start, int64_t& seq_end, int64_t& r0,
                                       int64_t& r1) const {
    if (!varlen) {
      int64_t b, c;
      if (idx32) {  // 32-bit division: a 64-bit one is a long subroutine on the GPU
        const uint32_t ii = static_cast<uint32_t>(i), tps = static_cast<uint32_t>(tiles_per_seq);
        const uint32_t b32 = ii / tps;
        b = b32;
        c = ii - b32 * tps;
      } else {
        b = i / tiles_per_seq;
        c = i - b * tiles_per_seq;
      }
      seq_start = b * seq_len;
      seq_end = seq_start + seq_len;
      r0 = seq_start + c * tile;
      r1 = r0 + tile < seq_end ? r0 + tile : seq_end;
      return r0 < r1;
    }
    const int64_t sid = ld_index(chunks, ch_i64, 2 * i);
    const int64_t c = ld_index(chunks, ch_i64, 2 * i + 1);
    if (sid < 0 || sid >= n_seqs || c < 0) return false;
    seq_start = ld_index(cu, cu_i64, sid);
    seq_end = ld_index(cu, cu_i64, sid + 1);
    if (seq_start < 0 || seq_end > n_tokens || seq_end <= seq_start) return false;
    if (c > (seq_end - seq_start) / chunk_size) return false;
    r0 = seq_start + c * chunk_size;
    r1 = r0 + chunk_size < seq_end ? r0 + chunk_size : seq_end;
    return r0 < r1;
  }
};

inline RowMap make_rowmap(const moc_problem& p, int32_t fixed_tile) {
  RowMap m;
  m.n_tokens = p.n_tokens;
  if (p.cu_seqlens != nullptr) {
    m.varlen = 1;
    m.cu = p.cu_seqlens;
    m.cu_i64 = p.cu_seqlens_dtype == MOC_INDEX_I64;
    m.n_seqs = p.n_seqs;
    m.chunks = p.chunk_indices;
    m.ch_i64 = p.chunk_indices_dtype == MOC_INDEX_I64;
    m.n_chunks = p.n_chunks;
    m.chunk_size = p.chunk_size;
  } else {
    m.batch = p.batch;
    m.seq_len = p.seq_len;
    m.tile = fixed_tile;
    m.tiles_per_seq = (p.seq_len + fixed_tile - 1) / fixed_tile;
    m.idx32 = p.batch * m.tiles_per_seq < (int64_t{1} << 31) ? 1 : 0;
    if (p.halo != nullptr) {
      m.halo = p.halo;
      m.hs0 = p.halo_strides[0];
      m.hs1 = p.halo_strides[1];
      m.hs2 = p.halo_strides[2];
      m.halo_S = p.kernel_size;
      m.halo_dt = p.x_dtype;
    }
  }
  return m;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Counts kernel launches for moc_launch_count(); call once per <<<>>> launch.
void note_launch(int n = 1);

// Records the last CUDA error for moc_last_cuda_error(); returns MOC_ERR_CUDA or MOC_OK.
int note_cuda(cudaError_t e);

}  // namespace moc
