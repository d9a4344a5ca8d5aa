// Generic CUDA-core MoC kernels.
//
// This path computes in true fp32 (the fp32 compute mode the reference only
// approximates with TF32 dots) and reproduces the bf16 rounding points of the
// reference's bf16 mode.  It serves every dtype mix, any K <= 128 and any S <= 64;
// the tensor-core path in moc_tc.cu takes over the bf16 shapes it supports.
//
// Reference semantics followed here:
//   forward      moc/kernels.py:36-142   y[t] = sum_s x[t-(S-1-s)] * sum_k a[t,k] w[k,s]
//   dx           moc/kernels.py:156-268  dx[t] = sum_s dz[t+S-1-s] * sum_k a[t+S-1-s,k] w[k,s]
//   dalpha/dbasis moc/kernels.py:282-426 m = dz * x_shift; da = m . w^T; dw = a^T . m
//   decode step  moc/kernels.py:442-550
#include <type_traits>

#include "moc_common.cuh"
#include "moc_internal.h"

namespace moc {
namespace {

constexpr int kSimtTile = 64;    // rows per fixed-length work item
constexpr int kSimtGroups = 32;  // token groups for the dbasis / dweight partial sums

template <typename XT>
struct ConvArgs {
  RowMap rm;
  int64_t D;
  int K, S;
  const XT* x;
  const void* alpha;
  int adt;
  const void* basis;
  int bdt;
  const XT* dy;
  const float* dz;  // fp32 dz = dy * silu'(pre) when the activation is on, else null
  XT* out;
  XT* dx;
  void* dalpha;
  float* partial;
  float* dz_out;
  int act;
  int64_t groups;
};

template <typename XT>
__device__ __forceinline__ float conv_pre(const ConvArgs<XT>& a, int64_t r, int64_t d, int64_t seq_start) {
  constexpr bool BF = std::is_same<XT, bf16>::value;
  float acc = 0.f;
  for (int s = 0; s < a.S; ++s) {
    const int64_t src = r - (a.S - 1 - s);
    float w = 0.f;
    for (int k = 0; k < a.K; ++k) {
      const float av = cround<BF>(ld_any(a.alpha, a.adt, r * a.K + k));
      const float bv = cround<BF>(ld_any(a.basis, a.bdt, (static_cast<int64_t>(k) * a.S + s) * a.D + d));
      w = fmaf(av, bv, w);
    }
    const float xv = src >= seq_start ? to_f32(a.x[src * a.D + d]) : a.rm.halo_at(seq_start, src, d);
    acc = fmaf(xv, w, acc);
  }
  return acc;
}

template <typename XT>
__device__ __forceinline__ float dz_at(const ConvArgs<XT>& a, int64_t r, int64_t d) {
  return a.dz != nullptr ? a.dz[r * a.D + d] : to_f32(a.dy[r * a.D + d]);
}

// grid (items, ceil(D/32)), block (32, 8): lane = channel, y = row stride.
template <typename XT>
__global__ void __launch_bounds__(256) k_fwd(ConvArgs<XT> a) {
  const int64_t d = static_cast<int64_t>(blockIdx.y) * 32 + threadIdx.x;
  int64_t ss, se, r0, r1;
  if (d >= a.D || !a.rm.item(blockIdx.x, ss, se, r0, r1)) return;
  for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y) {
    float v = conv_pre(a, r, d, ss);
    if (a.act) v = silu_f(v);
    a.out[r * a.D + d] = from_f32<XT>(v);
  }
}

// dz = dy * silu'(pre), pre recomputed in fp32.
template <typename XT>
__global__ void __launch_bounds__(256) k_dz(ConvArgs<XT> a) {
  const int64_t d = static_cast<int64_t>(blockIdx.y) * 32 + threadIdx.x;
  int64_t ss, se, r0, r1;
  if (d >= a.D || !a.rm.item(blockIdx.x, ss, se, r0, r1)) return;
  for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y) {
    const float pre = conv_pre(a, r, d, ss);
    a.dz_out[r * a.D + d] = to_f32(a.dy[r * a.D + d]) * dsilu_f(pre);
  }
}

template <typename XT>
__global__ void __launch_bounds__(256) k_dx(ConvArgs<XT> a) {
  constexpr bool BF = std::is_same<XT, bf16>::value;
  const int64_t d = static_cast<int64_t>(blockIdx.y) * 32 + threadIdx.x;
  int64_t ss, se, r0, r1;
  if (d >= a.D || !a.rm.item(blockIdx.x, ss, se, r0, r1)) return;
  for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y) {
    float acc = 0.f;
    for (int s = 0; s < a.S; ++s) {
      const int64_t u = r + (a.S - 1 - s);
      if (u >= se) continue;
      float w = 0.f;
      for (int k = 0; k < a.K; ++k) {
        const float av = cround<BF>(ld_any(a.alpha, a.adt, u * a.K + k));
        const float bv = cround<BF>(ld_any(a.basis, a.bdt, (static_cast<int64_t>(k) * a.S + s) * a.D + d));
        w = fmaf(av, bv, w);
      }
      acc = fmaf(dz_at(a, u, d), w, acc);
    }
    a.dx[r * a.D + d] = from_f32<XT>(acc);
  }
}

// One warp per token row reduces over all D channels and S taps; the butterfly
// shuffle reduction gives a fixed summation order, so dalpha is deterministic.
template <typename XT, int KMAX>
__global__ void __launch_bounds__(256) k_dalpha(ConvArgs<XT> a) {
  constexpr bool BF = std::is_same<XT, bf16>::value;
  int64_t ss, se, r0, r1;
  if (!a.rm.item(blockIdx.x, ss, se, r0, r1)) return;
  const int lane = threadIdx.x;
  for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y) {
    float acc[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) acc[k] = 0.f;
    for (int64_t d = lane; d < a.D; d += 32) {
      const float g = dz_at(a, r, d);
      for (int s = 0; s < a.S; ++s) {
        const int64_t src = r - (a.S - 1 - s);
        const float xv = src >= ss ? to_f32(a.x[src * a.D + d]) : a.rm.halo_at(ss, src, d);
        const float m = cround<BF>(g * xv);
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
          if (k < a.K) {
            const float bv = cround<BF>(ld_any(a.basis, a.bdt, (static_cast<int64_t>(k) * a.S + s) * a.D + d));
            acc[k] = fmaf(m, bv, acc[k]);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (k < a.K) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
      }
    }
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (k < a.K && (k & 31) == lane) st_any(a.dalpha, a.adt, r * a.K + k, acc[k]);
    }
  }
}

// grid (groups, ceil(D/32)), block (32, 8).  Group g owns items g, g+groups, ... and
// writes partial[g][k][s][d]; k_sum_partials adds the groups in a fixed order.
template <typename XT>
__global__ void __launch_bounds__(256) k_dbasis_partial(ConvArgs<XT> a) {
  constexpr bool BF = std::is_same<XT, bf16>::value;
  const int64_t g = blockIdx.x;
  const int64_t d = static_cast<int64_t>(blockIdx.y) * 32 + threadIdx.x;
  if (d >= a.D) return;
  const int KS = a.K * a.S;
  const int64_t n_items = a.rm.n_items();
  for (int p = threadIdx.y; p < KS; p += blockDim.y) {
    const int k = p / a.S;
    const int s = p - k * a.S;
    float acc = 0.f;
    for (int64_t i = g; i < n_items; i += a.groups) {
      int64_t ss, se, r0, r1;
      if (!a.rm.item(i, ss, se, r0, r1)) continue;
      for (int64_t r = r0; r < r1; ++r) {
        const int64_t src = r - (a.S - 1 - s);
        const float xv = src >= ss ? to_f32(a.x[src * a.D + d]) : a.rm.halo_at(ss, src, d);
        const float m = cround<BF>(dz_at(a, r, d) * xv);
        acc = fmaf(cround<BF>(ld_any(a.alpha, a.adt, r * a.K + k)), m, acc);
      }
    }
    a.partial[(g * KS + p) * a.D + d] = acc;
  }
}

// out[i] = sum_g partial[g][i], summed in increasing g.
__global__ void k_sum_partials(const float* __restrict__ partial, int64_t groups, int64_t n, void* out,
                               int out_dtype) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int64_t g = 0; g < groups; ++g) s += partial[g * n + i];
    st_any(out, out_dtype, i, s);
  }
}

// ------------------------------------------------------------------ decode step

template <typename XT>
__global__ void __launch_bounds__(128) k_step(int64_t D, int K, int S, const XT* __restrict__ x, const void* alpha,
                                              int adt, const void* basis, int bdt, XT* cache, int64_t cs0,
                                              int64_t cs1, int64_t cs2, XT* __restrict__ out, int act) {
  constexpr bool BF = std::is_same<XT, bf16>::value;
  const int64_t b = blockIdx.y;
  const int64_t d = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (d >= D) return;
  const XT xr = x[b * D + d];
  const float xv = to_f32(xr);
  XT* c = cache + b * cs0 + d * cs1;
  float acc = 0.f;
  for (int s = 0; s < S; ++s) {
    const float state = s == S - 1 ? xv : to_f32(c[static_cast<int64_t>(s + 1) * cs2]);
    float w = 0.f;
    for (int k = 0; k < K; ++k) {
      const float av = cround<BF>(ld_any(alpha, adt, b * K + k));
      const float bv = cround<BF>(ld_any(basis, bdt, (static_cast<int64_t>(k) * S + s) * D + d));
      // bf16 mode forms a*w in bf16 and sums in fp32 (moc/kernels.py:508-512)
      w += cround<BF>(av * bv);
    }
    acc = fmaf(state, w, acc);
  }
  if (act) acc = silu_f(acc);
  out[b * D + d] = from_f32<XT>(acc);
  for (int s = 0; s + 1 < S; ++s) c[static_cast<int64_t>(s) * cs2] = c[static_cast<int64_t>(s + 1) * cs2];
  c[static_cast<int64_t>(S - 1) * cs2] = xr;
}

// ------------------------------------------------------------------ router

// One warp per token: logits[k] = z[r,:] . w[k,:] in fp32, then softmax or exp.
template <int KMAX>
__global__ void __launch_bounds__(256) k_router_fwd(int64_t N, int64_t Dz, int K, int dt, int act, const void* z,
                                                    const void* w, void* alpha) {
  const int lane = threadIdx.x;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  if (r >= N) return;
  float acc[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) acc[k] = 0.f;
  for (int64_t c = lane; c < Dz; c += 32) {
    const float zv = ld_any(z, dt, r * Dz + c);
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) acc[k] = fmaf(zv, ld_any(w, dt, k * Dz + c), acc[k]);
  }
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    if (k < K) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
    }
  }
  float mx = 0.f, sum = 1.f;
  if (act == 0) {
    mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) mx = fmaxf(mx, acc[k]);
    sum = 0.f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) sum += expf(acc[k] - mx);
  }
  const float inv = 1.f / sum;
#pragma unroll
  for (int k = 0; k < KMAX; ++k)
    if (k < K && (k & 31) == lane) st_any(alpha, dt, r * K + k, expf(acc[k] - mx) * inv);
}

// dl[r,k] = alpha*(dalpha - sum_j alpha_j dalpha_j) (softmax) or alpha*dalpha (exp).
__global__ void k_router_dl(int64_t N, int K, int dt, int act, const void* alpha, const void* dalpha, int dadt,
                            float* dl) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= N) return;
  float dot = 0.f;
  if (act == 0)
    for (int k = 0; k < K; ++k) dot += ld_any(alpha, dt, r * K + k) * ld_any(dalpha, dadt, r * K + k);
  for (int k = 0; k < K; ++k)
    dl[r * K + k] = ld_any(alpha, dt, r * K + k) * (ld_any(dalpha, dadt, r * K + k) - dot);
}

// dz[r,c] = sum_k dl[r,k] w[k,c]; block (32, 8) = 8 rows.
template <int KMAX>
__global__ void __launch_bounds__(256) k_router_dz(int64_t N, int64_t Dz, int K, int dt, const float* dl,
                                                   const void* w, void* dz) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  if (r >= N) return;
  float g[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) g[k] = k < K ? dl[r * K + k] : 0.f;
  for (int64_t c = threadIdx.x; c < Dz; c += 32) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) acc = fmaf(g[k], ld_any(w, dt, k * Dz + c), acc);
    st_any(dz, dt, r * Dz + c, acc);
  }
}

// partial[g][k][c] = sum over rows of group g of dl[r,k] z[r,c]; grid (groups, ceil(Dz/32)).
__global__ void __launch_bounds__(256) k_router_dw_partial(int64_t N, int64_t Dz, int K, int dt, int64_t groups,
                                                           const float* dl, const void* z, float* partial) {
  const int64_t g = blockIdx.x;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * 32 + threadIdx.x;
  if (c >= Dz) return;
  const int64_t rows = (N + groups - 1) / groups;
  const int64_t r0 = g * rows;
  const int64_t r1 = r0 + rows < N ? r0 + rows : N;
  for (int k = threadIdx.y; k < K; k += blockDim.y) {
    float acc = 0.f;
    for (int64_t r = r0; r < r1; ++r) acc = fmaf(dl[r * K + k], ld_any(z, dt, r * Dz + c), acc);
    partial[(g * K + k) * Dz + c] = acc;
  }
}

// ------------------------------------------------------------------ chunk indices

// Single block: exclusive scan of per-sequence chunk counts, then each thread writes
// the (seq_id, chunk) pairs of its sequence (moc/ops.py:82-97 computes the same table).
// Rows past the last chunk (a table sized by an upper bound, so that the host never reads
// the offsets) are written as (-1, -1), which every kernel reads as an empty item.
__global__ void __launch_bounds__(1024) k_chunk_indices(const void* cu, int cu_i64, int64_t n_seqs, int chunk,
                                                        int32_t* out, int64_t n_chunks) {
  __shared__ int64_t warp_tot[32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t base = 0; base < n_seqs; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    int64_t cnt = 0;
    if (i < n_seqs) {
      const int64_t len = ld_index(cu, cu_i64, i + 1) - ld_index(cu, cu_i64, i);
      cnt = len > 0 ? (len + chunk - 1) / chunk : 0;
    }
    int64_t incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    int64_t before = 0;
    for (int w = 0; w < wid; ++w) before += warp_tot[w];
    const int64_t excl = carry + before + incl - cnt;
    for (int64_t j = 0; j < cnt; ++j) {
      const int64_t o = excl + j;
      if (o < n_chunks) {
        out[2 * o] = static_cast<int32_t>(i);
        out[2 * o + 1] = static_cast<int32_t>(j);
      }
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + cnt;
    __syncthreads();
  }
  for (int64_t o = carry + threadIdx.x; o < n_chunks; o += blockDim.x) {
    out[2 * o] = -1;
    out[2 * o + 1] = -1;
  }
}

template <typename Fn>
int dispatch_kmax(int K, Fn&& fn) {
  if (K <= 8) return fn(std::integral_constant<int, 8>{});
  if (K <= 16) return fn(std::integral_constant<int, 16>{});
  if (K <= 32) return fn(std::integral_constant<int, 32>{});
  if (K <= 64) return fn(std::integral_constant<int, 64>{});
  if (K <= 128) return fn(std::integral_constant<int, 128>{});
  return MOC_ERR_UNSUPPORTED_SHAPE;
}

template <typename XT>
ConvArgs<XT> conv_args(const moc_problem& p, const void* x, const void* alpha, const void* basis) {
  ConvArgs<XT> a{};
  a.rm = make_rowmap(p, kSimtTile);
  a.D = p.dim;
  a.K = p.n_bases;
  a.S = p.kernel_size;
  a.x = static_cast<const XT*>(x);
  a.alpha = alpha;
  a.adt = p.alpha_dtype;
  a.basis = basis;
  a.bdt = p.basis_dtype;
  a.act = p.activation;
  return a;
}

int64_t dbasis_groups(const RowMap& rm) {
  const int64_t n = rm.n_items();
  return n < kSimtGroups ? (n > 0 ? n : 1) : kSimtGroups;
}

template <typename XT>
int forward_t(const moc_problem& p, const void* x, const void* alpha, const void* basis, void* out,
              cudaStream_t st) {
  ConvArgs<XT> a = conv_args<XT>(p, x, alpha, basis);
  a.out = static_cast<XT*>(out);
  const int64_t items = a.rm.n_items();
  if (items == 0) return MOC_OK;
  dim3 grid(static_cast<unsigned>(items), static_cast<unsigned>(ceil_div(p.dim, 32)));
  k_fwd<XT><<<grid, dim3(32, 8), 0, st>>>(a);
  note_launch();
  return note_cuda(cudaGetLastError());
}

template <typename XT>
int backward_t(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy,
               void* dx, void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st) {
  ConvArgs<XT> a = conv_args<XT>(p, x, alpha, basis);
  a.dy = static_cast<const XT*>(dy);
  a.dx = static_cast<XT*>(dx);
  a.dalpha = dalpha;
  const int64_t items = a.rm.n_items();
  const int64_t groups = dbasis_groups(a.rm);
  a.groups = groups;
  const int64_t ksd = static_cast<int64_t>(p.n_bases) * p.kernel_size * p.dim;
  if (ws_bytes < simt_backward_ws(p)) return MOC_ERR_WORKSPACE_TOO_SMALL;
  char* wp = static_cast<char*>(ws);
  a.partial = reinterpret_cast<float*>(wp);
  wp += align_up(static_cast<size_t>(groups * ksd) * sizeof(float), 256);
  dim3 grid(static_cast<unsigned>(items > 0 ? items : 1), static_cast<unsigned>(ceil_div(p.dim, 32)));
  if (items > 0 && p.activation) {
    a.dz_out = reinterpret_cast<float*>(wp);
    k_dz<XT><<<grid, dim3(32, 8), 0, st>>>(a);
    note_launch();
    a.dz = a.dz_out;
  }
  if (items > 0 && dx != nullptr) {
    k_dx<XT><<<grid, dim3(32, 8), 0, st>>>(a);
    note_launch();
  }
  int rc = MOC_OK;
  if (items > 0) {
    rc = dispatch_kmax(p.n_bases, [&](auto km) {
      k_dalpha<XT, decltype(km)::value><<<static_cast<unsigned>(items), dim3(32, 8), 0, st>>>(a);
      note_launch();
      return MOC_OK;
    });
    if (rc != MOC_OK) return rc;
  }
  dim3 pgrid(static_cast<unsigned>(groups), static_cast<unsigned>(ceil_div(p.dim, 32)));
  k_dbasis_partial<XT><<<pgrid, dim3(32, 8), 0, st>>>(a);
  note_launch();
  const int64_t blocks = ceil_div(ksd, 256) < 4096 ? ceil_div(ksd, 256) : 4096;
  k_sum_partials<<<static_cast<unsigned>(blocks), 256, 0, st>>>(a.partial, groups, ksd, dbasis, p.basis_dtype);
  note_launch();
  return note_cuda(cudaGetLastError());
}

}  // namespace

int simt_forward(const moc_problem& p, const void* x, const void* alpha, const void* basis, void* out,
                 cudaStream_t st) {
  if (p.x_dtype == MOC_DTYPE_BF16) return forward_t<bf16>(p, x, alpha, basis, out, st);
  return forward_t<float>(p, x, alpha, basis, out, st);
}

size_t simt_backward_ws(const moc_problem& p) {
  const RowMap rm = make_rowmap(p, kSimtTile);
  const int64_t groups = dbasis_groups(rm);
  const int64_t ksd = static_cast<int64_t>(p.n_bases) * p.kernel_size * p.dim;
  size_t bytes = align_up(static_cast<size_t>(groups * ksd) * sizeof(float), 256);
  if (p.activation) bytes += align_up(static_cast<size_t>(p.n_tokens * p.dim) * sizeof(float), 256);
  return bytes;
}

int simt_backward(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy,
                  void* dx, void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (p.x_dtype == MOC_DTYPE_BF16)
    return backward_t<bf16>(p, x, alpha, basis, dy, dx, dalpha, dbasis, ws, ws_bytes, st);
  return backward_t<float>(p, x, alpha, basis, dy, dx, dalpha, dbasis, ws, ws_bytes, st);
}

int simt_step(int64_t B, int64_t D, int K, int S, int x_dtype, int a_dtype, int b_dtype, int act, const void* x,
              const void* alpha, const void* basis, void* cache, const int64_t cs[3], void* out, cudaStream_t st) {
  if (B == 0 || D == 0) return MOC_OK;
  dim3 grid(static_cast<unsigned>(ceil_div(D, 128)), static_cast<unsigned>(B));
  if (x_dtype == MOC_DTYPE_BF16)
    k_step<bf16><<<grid, 128, 0, st>>>(D, K, S, static_cast<const bf16*>(x), alpha, a_dtype, basis, b_dtype,
                                       static_cast<bf16*>(cache), cs[0], cs[1], cs[2], static_cast<bf16*>(out), act);
  else
    k_step<float><<<grid, 128, 0, st>>>(D, K, S, static_cast<const float*>(x), alpha, a_dtype, basis, b_dtype,
                                        static_cast<float*>(cache), cs[0], cs[1], cs[2], static_cast<float*>(out),
                                        act);
  note_launch();
  return note_cuda(cudaGetLastError());
}

int simt_router_forward(int64_t N, int64_t Dz, int K, int dtype, int act, const void* z, const void* w,
                        void* alpha, cudaStream_t st) {
  if (N == 0) return MOC_OK;
  const unsigned blocks = static_cast<unsigned>(ceil_div(N, 8));
  int rc = dispatch_kmax(K, [&](auto km) {
    k_router_fwd<decltype(km)::value><<<blocks, dim3(32, 8), 0, st>>>(N, Dz, K, dtype, act, z, w, alpha);
    note_launch();
    return MOC_OK;
  });
  if (rc != MOC_OK) return rc;
  return note_cuda(cudaGetLastError());
}

static int64_t router_groups(int64_t N) {
  const int64_t g = ceil_div(N, 512);
  return g < 1 ? 1 : (g > 64 ? 64 : g);
}

size_t simt_router_backward_ws(int64_t N, int64_t Dz, int K) {
  return align_up(static_cast<size_t>(N * K) * sizeof(float), 256) +
         align_up(static_cast<size_t>(router_groups(N) * K * Dz) * sizeof(float), 256);
}

int simt_router_backward(int64_t N, int64_t Dz, int K, int dtype, int act, const void* z, const void* w,
                         const void* alpha, const void* dalpha, int da_dtype, void* dz, void* dw, void* ws,
                         size_t ws_bytes, cudaStream_t st) {
  if (ws_bytes < simt_router_backward_ws(N, Dz, K)) return MOC_ERR_WORKSPACE_TOO_SMALL;
  float* dl = static_cast<float*>(ws);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                            align_up(static_cast<size_t>(N * K) * sizeof(float), 256));
  const int64_t groups = router_groups(N);
  if (N > 0) {
    k_router_dl<<<static_cast<unsigned>(ceil_div(N, 256)), 256, 0, st>>>(N, K, dtype, act, alpha, dalpha,
                                                                                 da_dtype, dl);
    note_launch();
  }
  if (N > 0 && dz != nullptr) {
    int rc = dispatch_kmax(K, [&](auto km) {
      k_router_dz<decltype(km)::value><<<static_cast<unsigned>(ceil_div(N, 8)), dim3(32, 8), 0, st>>>(
          N, Dz, K, dtype, dl, w, dz);
      note_launch();
      return MOC_OK;
    });
    if (rc != MOC_OK) return rc;
  }
  if (dw != nullptr) {
    const int64_t n = static_cast<int64_t>(K) * Dz;
    if (N > 0) {
      dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(ceil_div(Dz, 32)));
      k_router_dw_partial<<<grid, dim3(32, 8), 0, st>>>(N, Dz, K, dtype, groups, dl, z, partial);
      note_launch();
    } else {
      cudaMemsetAsync(partial, 0, static_cast<size_t>(n) * sizeof(float), st);
    }
    const int64_t blocks = ceil_div(n, 256) < 4096 ? ceil_div(n, 256) : 4096;
    k_sum_partials<<<static_cast<unsigned>(blocks), 256, 0, st>>>(partial, N > 0 ? groups : 1, n, dw, dtype);
    note_launch();
  }
  return note_cuda(cudaGetLastError());
}

int build_chunk_indices(const void* cu, int cu_i64, int64_t n_seqs, int chunk, int32_t* out, int64_t n_chunks,
                        cudaStream_t st) {
  if (n_chunks == 0) return MOC_OK;
  k_chunk_indices<<<1, 1024, 0, st>>>(cu, cu_i64, n_seqs, chunk, out, n_chunks);
  note_launch();
  return note_cuda(cudaGetLastError());
}

}  // namespace moc
