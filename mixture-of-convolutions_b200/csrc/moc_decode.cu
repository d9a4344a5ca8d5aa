// Fused decode step for several MoC modules that share the routing input z (the q / k / v
// convolutions of an attention block, reference README.md:120-129), bf16.
//
// Two launches for all modules instead of a router GEMM, an activation and an update
// kernel per module:
//   k_dec_router  a cluster of 8 CTAs per (16 tokens, module).  CTA r of the cluster
//                 streams z and the module's router weight for the 512-column chunks
//                 r, r+8, ... through a 2-stage cp.async ring; its 8 warps own 64 columns
//                 of a chunk each and accumulate the 16 x 16 logit tile with mma.sync
//                 (bf16 -> fp32).  The partial tiles are added in shared memory, then CTA 0
//                 adds the 8 CTAs' tiles through distributed shared memory in rank order
//                 and applies softmax / exp per token over 16 lanes (moc/api.py:383-388).
//   k_dec_update  CTA = (32 channels of one module, 16 tokens), warp = 8 channels.  One
//                 mma.sync per tap forms W_s = alpha . basis_s for the warp's 16 tokens x 8
//                 channels (bf16 products exact, fp32 sums: the rounding of the reference's
//                 bf16 forward, moc/kernels.py:125-130; its decode kernel rounds each product
//                 to bf16 first, moc/kernels.py:466-513, a difference far inside the bf16
//                 tolerance).  Then y = [silu](sum_s state_s * W_s) and each channel's
//                 cache row (S contiguous slots) is shifted and x appended
//                 (moc/kernels.py:522-550).  All loads of a warp are issued before the math.
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
constexpr int kDecRouterSmem = 2 * kDecStageBytes + 9 * kDecTok * kDecKP * 4;
constexpr int kDecCluster = 8;               // CTAs per router cluster (split of z_dim)
constexpr int kUpdTok = 16;                  // tokens per update CTA (MMA M)
constexpr int kUpdThreads = 128;             // 4 warps x 8 channels (MMA N)
constexpr int kUpdCh = 32;                   // channels per update CTA

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

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

// fp32 at shared address `addr` of this CTA, read from CTA `rank` of the cluster
__device__ __forceinline__ float ld_dsmem(uint32_t addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

__global__ void __cluster_dims__(kDecCluster, 1, 1) __launch_bounds__(256)
    k_dec_router(const __grid_constant__ DecArgs a) {
  extern __shared__ __align__(128) char smem[];
  float* red = reinterpret_cast<float*>(smem + 2 * kDecStageBytes);  // [8 warps][16 tokens][16 bases]
  float* part = red + 8 * kDecTok * kDecKP;                            // [16 tokens][16 bases]: this CTA's sum
  const DecModule& mod = a.m[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x / kDecCluster) * kDecTok;
  const int n_chunks = static_cast<int>((a.Dz + kDecCols - 1) / kDecCols);

  auto load = [&](int c, int st) {
    char* base = smem + st * kDecStageBytes;
    const int64_t col0 = static_cast<int64_t>(c) * kDecCols;
    for (int idx = threadIdx.x; idx < kDecStageRows * (kDecCols / 8); idx += 256) {
      const int row = idx / (kDecCols / 8), piece = idx - row * (kDecCols / 8);
      const int64_t col = col0 + piece * 8;
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
      cp_async16(smem_addr(base + row * kDecPitch + piece * 16), ok ? src : a.z, ok ? 16u : 0u);
    }
  };

  // this CTA's chunks: rank, rank + 8, ...
  float acc[2][4] = {};
  int n = 0;
  if (static_cast<int>(rank) < n_chunks) {
    load(rank, 0);
    cp_async_commit();
  }
  for (int c = rank; c < n_chunks; c += kDecCluster, ++n) {
    if (c + kDecCluster < n_chunks) {
      load(c + kDecCluster, (n + 1) & 1);  // the stage of this CTA's previous chunk, released below
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t zs = smem_addr(smem + (n & 1) * kDecStageBytes);
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
  part[t * kDecKP + k] = l;
  cluster_sync_all();  // every CTA's partial tile is visible to the cluster
  if (rank == 0) {
    const uint32_t addr = smem_addr(part + t * kDecKP + k);
    l = 0.f;
#pragma unroll
    for (uint32_t rr = 0; rr < kDecCluster; ++rr) l += ld_dsmem(addr, rr);
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
  cluster_sync_all();  // CTA 0 has read every partial tile before any CTA exits
}

// One channel's cache row: S contiguous bf16 slots (2*S bytes: 4-byte aligned for even S).
template <int S>
struct CacheRow {
  static constexpr int kWords = (S + 1) / 2;
  uint32_t w[kWords];  // slot i in bits 16*(i&1) of word i/2
  __device__ __forceinline__ uint32_t slot(int i) const { return (w[i >> 1] >> (16 * (i & 1))) & 0xffffu; }
};
template <int S>
__device__ __forceinline__ CacheRow<S> load_row(const bf16* p) {
  CacheRow<S> r;
  if constexpr (S == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    r.w[0] = u.x, r.w[1] = u.y;
  } else if constexpr (S == 2) {
    r.w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int i = 0; i < CacheRow<S>::kWords; ++i)
      r.w[i] = h[2 * i] | (2 * i + 1 < S ? (uint32_t(h[2 * i + 1]) << 16) : 0u);
  }
  return r;
}
// Writes slots 1..S-1 of `old` to slots 0..S-2 and x to slot S-1.
template <int S>
__device__ __forceinline__ void store_shifted(bf16* p, const CacheRow<S>& old, uint32_t x) {
  uint32_t v[S];
#pragma unroll
  for (int i = 0; i + 1 < S; ++i) v[i] = old.slot(i + 1);
  v[S - 1] = x;
  if constexpr (S == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(v[0] | (v[1] << 16), v[2] | (v[3] << 16));
  } else if constexpr (S == 2) {
    *reinterpret_cast<uint32_t*>(p) = v[0] | (v[1] << 16);
  } else {
#pragma unroll
    for (int i = 0; i < S; ++i) reinterpret_cast<uint16_t*>(p)[i] = static_cast<uint16_t>(v[i]);
  }
}

template <int S>
__global__ void __launch_bounds__(kUpdThreads) k_dec_update(const __grid_constant__ DecArgs a) {
  int m = 0;
  while (m + 1 < a.n_mod && static_cast<int>(blockIdx.x) >= a.blk_prefix[m + 1]) ++m;
  const DecModule& mod = a.m[m];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t cw = static_cast<int64_t>(static_cast<int>(blockIdx.x) - a.blk_prefix[m]) * kUpdCh + warp * 8;
  const int64_t b0 = static_cast<int64_t>(blockIdx.y) * kUpdTok;
  if (cw >= mod.D) return;  // whole warp
  const uint16_t* al = reinterpret_cast<const uint16_t*>(mod.alpha);
  const uint16_t* bs = reinterpret_cast<const uint16_t*>(mod.basis);
  const uint16_t* xs = reinterpret_cast<const uint16_t*>(mod.x);

  // every load of the warp's tile first (one round trip): B operand = basis of channel
  // cw + g (n) and bases 2q.. / 2q+8.. (k) per tap; A operand = alpha of tokens b0 + g,
  // b0 + g + 8 and the same bases; x and cache rows of (tokens b0+g, b0+g+8) x
  // (channels cw+2q, cw+2q+1).  Bases past K, channels past D and tokens past B read 0.
  auto ld = [](const uint16_t* p, int64_t i, bool ok) -> uint32_t { return ok ? p[i] : 0u; };
  uint32_t bf[S][2];
  {
    const int64_t ch = cw + g;
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = 2 * q + 8 * j;
        bf[s][j] = ld(bs, (static_cast<int64_t>(k) * S + s) * mod.D + ch, ch < mod.D && k < mod.K) |
                   (ld(bs, (static_cast<int64_t>(k + 1) * S + s) * mod.D + ch, ch < mod.D && k + 1 < mod.K) << 16);
      }
  }
  uint32_t af[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t b = b0 + g + 8 * (r & 1);
    const int k = 2 * q + 8 * (r >> 1);
    af[r] = ld(al, b * mod.K + k, b < a.B && k < mod.K) | (ld(al, b * mod.K + k + 1, b < a.B && k + 1 < mod.K) << 16);
  }
  uint32_t xv[2][2];
  CacheRow<S> cr[2][2];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t b = b0 + g + 8 * h, ch = cw + 2 * q + e;
      const bool ok = b < a.B && ch < mod.D;
      xv[h][e] = ld(xs, b * mod.D + ch, ok);
#pragma unroll
      for (int i = 0; i < CacheRow<S>::kWords; ++i) cr[h][e].w[i] = 0;
      if (ok) cr[h][e] = load_row<S>(mod.cache + (b * mod.D + ch) * S);
    }

  // W_s = alpha . basis_s for 16 tokens x 8 channels per tap (fp32 accumulate), then
  // y = sum_s state_s * W_s with state_s = cache slot s+1, x for the newest tap
  float acc[2][2] = {};
#pragma unroll
  for (int s = 0; s < S; ++s) {
    float w[4];
    mma_bf16_z(w, af, bf[s][0], bf[s][1]);  // w[2h + e]: token b0+g+8h, channel cw+2q+e
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t st = s == S - 1 ? xv[h][e] : cr[h][e].slot(s + 1);
        acc[h][e] = fmaf(__uint_as_float(st << 16), w[2 * h + e], acc[h][e]);
      }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t b = b0 + g + 8 * h, ch = cw + 2 * q + e;
      if (b < a.B && ch < mod.D) {
        const float v = mod.act ? silu_f(acc[h][e]) : acc[h][e];
        mod.out[b * mod.D + ch] = __float2bfloat16_rn(v);
        store_shifted<S>(mod.cache + (b * mod.D + ch) * S, cr[h][e], xv[h][e]);
      }
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
  k_dec_router<<<dim3(static_cast<unsigned>(ceil_div(B, kDecTok) * kDecCluster), static_cast<unsigned>(n)), 256,
                 kDecRouterSmem, st>>>(a);
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
