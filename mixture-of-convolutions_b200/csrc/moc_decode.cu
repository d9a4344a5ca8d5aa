// Fused decode step for several MoC modules that share the routing input z (the q / k / v
// convolutions of an attention block, reference README.md:120-129), bf16.
//
// Two launches for all modules instead of a router GEMM, an activation and an update
// kernel per module:
//   k_dec_router  CTA = (16 tokens, module).  z and the module's router weight stream
//                 through a 2-stage cp.async ring in 512-column chunks; each of the 8
//                 warps owns 64 columns of a chunk and accumulates the 16 x 16 logit tile
//                 with mma.sync (bf16 -> fp32); the 8 partial tiles are added in shared
//                 memory in a fixed order and softmax / exp is applied per token over 16
//                 lanes (moc/api.py:383-388).
//   k_dec_update  CTA = (256 channels of one module, 4 tokens), thread = channel pair.
//                 The thread's basis column (K x S bf16 pairs) stays in registers across
//                 the tokens; per token W_s = sum_k bf16(alpha_k * basis_ks) in fp32 (the
//                 reference's bf16 decode forms the products in bf16, moc/kernels.py:
//                 466-513), y = [silu](sum_s state_s * W_s), then the cache row of both
//                 channels (S contiguous slots each) is shifted and x appended in one
//                 vector store (moc/kernels.py:522-550).
#include <algorithm>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_mma.cuh"

namespace moc {

namespace {

constexpr int kDecTok = 16;                  // tokens per router CTA (MMA M)
constexpr int kDecCols = 512;                // z columns per staged chunk
constexpr int kDecPitch = kDecCols * 2 + 16; // smem row pitch in bytes (16 B pad: conflict-free ldmatrix)
constexpr int kDecKP = 16;                   // bases per module, padded (MMA N = 2 x 8)
constexpr int kDecStageRows = kDecTok + kDecKP;
constexpr int kDecStageBytes = kDecStageRows * kDecPitch;
constexpr int kDecRouterSmem = 2 * kDecStageBytes + 8 * kDecTok * kDecKP * 4;
constexpr int kUpdTok = 4;                   // tokens per update CTA
constexpr int kUpdThreads = 128;
constexpr int kUpdCh = 2 * kUpdThreads;      // channels per update CTA

struct DecModule {
  const bf16* w;
  const bf16* basis;
  const bf16* x;
  bf16* cache;
  bf16* alpha;
  bf16* out;
  int64_t D;
  int K, act, ract;
};

struct DecArgs {
  DecModule m[MOC_DECODE_MAX_MODULES];
  int n_mod;
  int64_t B, Dz;
  const bf16* z;
  int blk_prefix[MOC_DECODE_MAX_MODULES + 1];  // update-kernel channel blocks, prefix sums over modules
};

__device__ __forceinline__ int lm_row_d(int lane) { return (lane & 7) + ((lane >> 3) & 1) * 8; }
__device__ __forceinline__ int lm_col_d(int lane) { return (lane >> 4) * 8; }

__global__ void __launch_bounds__(256) k_dec_router(const __grid_constant__ DecArgs a) {
  extern __shared__ __align__(128) char smem[];
  float* red = reinterpret_cast<float*>(smem + 2 * kDecStageBytes);  // [8 warps][16 tokens][16 bases]
  const DecModule& mod = a.m[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * kDecTok;
  const int n_chunks = static_cast<int>((a.Dz + kDecCols - 1) / kDecCols);

  auto load = [&](int c, int st) {
    char* base = smem + st * kDecStageBytes;
    const int64_t col0 = static_cast<int64_t>(c) * kDecCols;
    for (int idx = threadIdx.x; idx < kDecStageRows * (kDecCols / 8); idx += 256) {
      const int row = idx / (kDecCols / 8), part = idx - row * (kDecCols / 8);
      const int64_t col = col0 + part * 8;
      const bf16* src;
      bool ok;
      if (row < kDecTok) {
        const int64_t t = tok0 + row;
        ok = t < a.B && col < a.Dz;
        src = a.z + t * a.Dz + col;
      } else {
        const int k = row - kDecTok;
        ok = k < mod.K && col < a.Dz;
        src = mod.w + static_cast<int64_t>(k) * a.Dz + col;
      }
      cp_async16(smem_addr(base + row * kDecPitch + part * 16), ok ? src : a.z, ok ? 16u : 0u);
    }
  };

  float acc[2][4] = {};
  load(0, 0);
  cp_async_commit();
  for (int c = 0; c < n_chunks; ++c) {
    if (c + 1 < n_chunks) {
      load(c + 1, (c + 1) & 1);  // the stage of chunk c-1, released by the barrier below
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t zs = smem_addr(smem + (c & 1) * kDecStageBytes);
    const uint32_t ws = zs + kDecTok * kDecPitch;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int col = warp * 64 + kk * 16;
      uint32_t af[4], bf[4];
      ldsm_x4(zs + lm_row_d(lane) * kDecPitch + (col + lm_col_d(lane)) * 2, af);
      ldsm_x4(ws + ((lane & 7) + (lane >> 4) * 8) * kDecPitch + (col + ((lane >> 3) & 1) * 8) * 2, bf);
      mma_bf16(acc[0], af, bf[0], bf[1]);
      mma_bf16(acc[1], af, bf[2], bf[3]);
    }
    __syncthreads();
  }

  // acc[nt][2h + e] = partial logit (token g + 8h, base 8nt + 2q + e) of this warp's columns
  const int g = lane >> 2, q = lane & 3;
  float* r = red + warp * kDecTok * kDecKP;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h)
      *reinterpret_cast<float2*>(r + (g + 8 * h) * kDecKP + nt * 8 + 2 * q) =
          make_float2(acc[nt][2 * h], acc[nt][2 * h + 1]);
  __syncthreads();
  const int t = threadIdx.x >> 4, k = threadIdx.x & 15;  // 16 lanes per token
  float l = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) l += red[w * kDecTok * kDecKP + t * kDecKP + k];
  float v;
  if (mod.ract == 0) {
    float mx = k < mod.K ? l : -INFINITY;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e = k < mod.K ? expf(l - mx) : 0.f;
    float sum = e;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    v = e * (1.f / sum);
  } else {
    v = expf(l);
  }
  const int64_t tok = tok0 + t;
  if (tok < a.B && k < mod.K) mod.alpha[tok * mod.K + k] = __float2bfloat16_rn(v);
}

// Cache row of a channel pair: 2*S contiguous bf16 (channel d: slots 0..S-1, then d+1),
// moved as S 32-bit words.
template <int S>
__device__ __forceinline__ void load_pair_row(const bf16* p, uint32_t (&w)[S]) {
  if constexpr (S == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
  } else if constexpr (S == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x, w[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < S; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
  }
}

template <int S>
__device__ __forceinline__ void store_pair_row(bf16* p, const uint32_t (&w)[S]) {
  if constexpr (S == 4) {
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if constexpr (S == 2) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int i = 0; i < S; ++i) reinterpret_cast<uint32_t*>(p)[i] = w[i];
  }
}

// element e (0 .. 2S-1) of a pair row
template <int S>
__device__ __forceinline__ uint32_t pair_elem(const uint32_t (&w)[S], int e) {
  return (e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu);
}

template <int S>
__global__ void __launch_bounds__(kUpdThreads) k_dec_update(const __grid_constant__ DecArgs a) {
  __shared__ uint32_t aa[kUpdTok][kDecKP];  // alpha of (token, base) duplicated into both bf16 halves
  int m = 0;
  while (m + 1 < a.n_mod && static_cast<int>(blockIdx.x) >= a.blk_prefix[m + 1]) ++m;
  const DecModule& mod = a.m[m];
  const int64_t d = static_cast<int64_t>(static_cast<int>(blockIdx.x) - a.blk_prefix[m]) * kUpdCh + 2 * threadIdx.x;
  const int64_t b0 = static_cast<int64_t>(blockIdx.y) * kUpdTok;
  for (int i = threadIdx.x; i < kUpdTok * kDecKP; i += kUpdThreads) {
    const int t = i / kDecKP, k = i - t * kDecKP;
    const int64_t b = b0 + t;
    uint32_t v = 0;
    if (b < a.B && k < mod.K) {
      const uint32_t h = reinterpret_cast<const uint16_t*>(mod.alpha)[b * mod.K + k];
      v = h | (h << 16);
    }
    aa[t][k] = v;
  }
  __syncthreads();
  if (d >= mod.D) return;

  uint32_t bw[kDecKP][S];  // basis pairs (channels d, d+1) of base k, tap s
#pragma unroll
  for (int k = 0; k < kDecKP; ++k)
#pragma unroll
    for (int s = 0; s < S; ++s)
      bw[k][s] = k < mod.K ? *reinterpret_cast<const uint32_t*>(mod.basis + (static_cast<int64_t>(k) * S + s) * mod.D + d)
                           : 0u;

#pragma unroll 1
  for (int t = 0; t < kUpdTok; ++t) {
    const int64_t b = b0 + t;
    if (b >= a.B) break;
    const uint32_t xv = *reinterpret_cast<const uint32_t*>(mod.x + b * mod.D + d);
    bf16* crow = mod.cache + (b * mod.D + d) * S;
    uint32_t cw[S];
    load_pair_row<S>(crow, cw);
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      float w0 = 0.f, w1 = 0.f;
#pragma unroll
      for (int k = 0; k < kDecKP; ++k) {
        const uint32_t p = hmul2_bf16(aa[t][k], bw[k][s]);
        w0 += bf_lo(p);
        w1 += bf_hi(p);
      }
      // state s: cache slot s+1, or x for the newest tap
      const float st0 = s == S - 1 ? bf_lo(xv) : __uint_as_float(pair_elem<S>(cw, s + 1) << 16);
      const float st1 = s == S - 1 ? bf_hi(xv) : __uint_as_float(pair_elem<S>(cw, S + s + 1) << 16);
      acc0 = fmaf(st0, w0, acc0);
      acc1 = fmaf(st1, w1, acc1);
    }
    if (mod.act) {
      acc0 = silu_f(acc0);
      acc1 = silu_f(acc1);
    }
    *reinterpret_cast<uint32_t*>(mod.out + b * mod.D + d) = pack_bf16(acc0, acc1);
    // shifted row: channel d = [slots 1..S-1, x_d], channel d+1 likewise
    uint32_t nw[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      uint32_t e2[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int e = 2 * i + j;       // new element index in the pair row
        const int ch = e / S, slot = e - ch * S;
        e2[j] = slot == S - 1 ? (ch == 0 ? (xv & 0xffffu) : (xv >> 16)) : pair_elem<S>(cw, ch * S + slot + 1);
      }
      nw[i] = e2[0] | (e2[1] << 16);
    }
    store_pair_row<S>(crow, nw);
  }
}

int g_dec_sm_configured[64];

}  // namespace

int decode_step_multi(int n, const moc_decode_module* mods, int64_t B, int64_t Dz, const void* z, cudaStream_t st) {
  DecArgs a{};
  a.n_mod = n;
  a.B = B;
  a.Dz = Dz;
  a.z = static_cast<const bf16*>(z);
  const int S = mods[0].kernel_size;
  a.blk_prefix[0] = 0;
  for (int i = 0; i < n; ++i) {
    DecModule& m = a.m[i];
    m.w = static_cast<const bf16*>(mods[i].weight);
    m.basis = static_cast<const bf16*>(mods[i].basis);
    m.x = static_cast<const bf16*>(mods[i].x);
    m.cache = static_cast<bf16*>(mods[i].cache);
    m.alpha = static_cast<bf16*>(mods[i].alpha);
    m.out = static_cast<bf16*>(mods[i].out);
    m.D = mods[i].dim;
    m.K = mods[i].n_bases;
    m.act = mods[i].activation;
    m.ract = mods[i].router_act;
    a.blk_prefix[i + 1] = a.blk_prefix[i] + static_cast<int>(ceil_div(m.D, kUpdCh));
  }
  if (B == 0) return MOC_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return note_cuda(e);
  if (dev < 0 || dev >= 64 || !g_dec_sm_configured[dev]) {
    e = cudaFuncSetAttribute(k_dec_router, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecRouterSmem);
    if (e != cudaSuccess) return note_cuda(e);
    if (dev >= 0 && dev < 64) g_dec_sm_configured[dev] = 1;
  }
  k_dec_router<<<dim3(static_cast<unsigned>(ceil_div(B, kDecTok)), static_cast<unsigned>(n)), 256, kDecRouterSmem,
                 st>>>(a);
  note_launch();
  e = cudaGetLastError();
  if (e != cudaSuccess) return note_cuda(e);
  const dim3 grid(static_cast<unsigned>(a.blk_prefix[n]), static_cast<unsigned>(ceil_div(B, kUpdTok)));
  switch (S) {
    case 1: k_dec_update<1><<<grid, kUpdThreads, 0, st>>>(a); break;
    case 2: k_dec_update<2><<<grid, kUpdThreads, 0, st>>>(a); break;
    case 3: k_dec_update<3><<<grid, kUpdThreads, 0, st>>>(a); break;
    case 4: k_dec_update<4><<<grid, kUpdThreads, 0, st>>>(a); break;
    default: return MOC_ERR_UNSUPPORTED_SHAPE;
  }
  note_launch();
  return note_cuda(cudaGetLastError());
}

}  // namespace moc
