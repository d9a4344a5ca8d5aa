// Fused decode step for several MoC modules that share the routing input z (the q / k / v
// convolutions of an attention block, reference README.md:120-129), bf16.
//
// Two launches for all modules instead of a router GEMM, an activation and an update
// kernel per module:
//   k_dec_router  a cluster of 8 CTAs per (16 tokens, module).  CTA r of the cluster
//                 streams z and the module's router weight for the 512-column chunks
//                 r, r+8, ... through a 2-stage cp.async ring; its 8 warps own 64 columns
//                 of a chunk each and accumulate the 16 x 16 logit tile with mma.sync
//                 (bf16 -> fp32).  The partial tiles are added in shared memory, every CTA
//                 stores its tile into CTA 0's shared memory (distributed shared memory),
//                 and CTA 0 adds the 8 tiles in rank order and applies softmax / exp per
//                 token over 16 lanes (moc/api.py:383-388).
//   k_dec_update  CTA = (128 channels of one module, 16 tokens), launched as a programmatic
//                 dependent of the router: the basis slice, x and cache tiles arrive with
//                 16-byte copies while the router still runs, alpha once it has finished; per tap, one ldmatrix of
//                 the basis and two mma.sync per warp form W_s = alpha . basis_s for 16
//                 tokens x 16 channels (bf16 products exact, fp32 sums: the rounding of the
//                 reference's bf16 forward, moc/kernels.py:125-130; its decode kernel rounds
//                 each product to bf16 first, moc/kernels.py:466-513, a difference far inside
//                 the bf16 tolerance).  Then y = [silu](sum_s state_s * W_s), the cache rows
//                 are shifted in shared memory with x appended (moc/kernels.py:522-550),
//                 and y and the cache tile leave with 16-byte stores.
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
constexpr int kDecCluster = 8;               // CTAs per router cluster (split of z_dim)
constexpr int kDecRouterSmem = 2 * kDecStageBytes + (8 + kDecCluster) * kDecTok * kDecKP * 4;
constexpr int kUpdTok = 16;                  // tokens per update CTA (MMA M)
constexpr int kUpdThreads = 256;             // 8 warps x 16 channels (two MMA n-tiles)
constexpr int kUpdCh = 128;                  // channels per update CTA
constexpr int kUpdBasisPitch = kUpdCh * 2 + 16;  // padded rows: conflict-free ldmatrix
constexpr int kUpdAlphaPitch = 48;
constexpr int kUpdWPitch = kUpdCh * 4 + 16;     // fp32 W rows, padded

template <int S>
struct UpdLayout {
  static constexpr int basis = S * kDecKP * kUpdBasisPitch;
  static constexpr int alpha = kUpdTok * kUpdAlphaPitch;
  static constexpr int x = kUpdTok * kUpdCh * 2;
  static constexpr int cache = kUpdTok * kUpdCh * S * 2;
  static constexpr int w = S * kUpdTok * kUpdWPitch;
  static constexpr int total = basis + alpha + x + cache + w;
};

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

// Programmatic dependent launch: the router lets the update grid start at once; the update
// kernel stages everything that does not depend on the router (basis, x, cache) and then
// waits for the router grid's completion (and its alpha) before reading alpha.  Without the
// launch attribute both are no-ops and the kernels run one after the other.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

// Stores v at shared address `addr` (this CTA's layout) of CTA `rank` of the cluster.
__device__ __forceinline__ void st_dsmem(uint32_t addr, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(addr), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;\n" ::"r"(remote), "f"(v) : "memory");
}

__global__ void __cluster_dims__(kDecCluster, 1, 1) __launch_bounds__(256)
    k_dec_router(const __grid_constant__ DecArgs a) {
  extern __shared__ __align__(128) char smem[];
  float* red = reinterpret_cast<float*>(smem + 2 * kDecStageBytes);  // [8 warps][16 tokens][16 bases]
  float* part = red + 8 * kDecTok * kDecKP;  // [8 ranks][16 tokens][16 bases]: the cluster's CTA sums (rank 0's)
  const DecModule& mod = a.m[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x / kDecCluster) * kDecTok;
  const int n_chunks = static_cast<int>((a.Dz + kDecCols - 1) / kDecCols);
  griddep_launch_dependents();

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
  // every CTA puts its tile into rank 0's shared memory; rank 0 adds them in rank order
  st_dsmem(smem_addr(part + (rank * kDecTok + t) * kDecKP + k), 0, l);
  cluster_sync_all();
  if (rank == 0) {
    l = 0.f;
#pragma unroll
    for (int rr = 0; rr < kDecCluster; ++rr) l += part[(rr * kDecTok + t) * kDecKP + k];
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
}

template <int S>
__global__ void __launch_bounds__(kUpdThreads) k_dec_update(const __grid_constant__ DecArgs a) {
  // tiles of this CTA's 16 tokens x 128 channels, loaded with 16-byte copies (dynamic
  // shared memory, UpdLayout<S>)
  extern __shared__ __align__(16) char upd_smem[];
  using UL = UpdLayout<S>;
  char* basis_s = upd_smem;                // [tap][base][128 ch], bases past K zero
  char* alpha_s = basis_s + UL::basis;     // [token][16 bases]
  char* x_s = alpha_s + UL::alpha;         // [token][128 ch]; y replaces x in place
  char* cache_s = x_s + UL::x;             // [token][128 ch][S]
  char* w_s = cache_s + UL::cache;         // [tap][token][128 ch] fp32
  char* y_s = x_s;
  int m = 0;
  while (m + 1 < a.n_mod && static_cast<int>(blockIdx.x) >= a.blk_prefix[m + 1]) ++m;
  const DecModule& mod = a.m[m];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t c0 = static_cast<int64_t>(static_cast<int>(blockIdx.x) - a.blk_prefix[m]) * kUpdCh;
  const int64_t b0 = static_cast<int64_t>(blockIdx.y) * kUpdTok;
  const int nch = static_cast<int>(mod.D - c0 < kUpdCh ? mod.D - c0 : kUpdCh);  // multiple of 8
  const int ntok = static_cast<int>(a.B - b0 < kUpdTok ? a.B - b0 : kUpdTok);

  // ---- loads (16-byte pieces; missing channels, tokens and bases become zeros)
  constexpr int kPieces = kUpdCh / 8;  // 16-byte pieces per 64-channel row
  for (int i = threadIdx.x; i < S * kDecKP * kPieces; i += kUpdThreads) {
    const int row = i / kPieces, p = i - row * kPieces;  // row = s * 16 + k
    const int s = row / kDecKP, k = row - s * kDecKP;
    const bool ok = k < mod.K && p * 8 < nch;
    cp_async16(smem_addr(basis_s + row * kUpdBasisPitch + p * 16),
               ok ? mod.basis + (static_cast<int64_t>(k) * S + s) * mod.D + c0 + p * 8 : mod.basis, ok ? 16u : 0u);
  }
  for (int i = threadIdx.x; i < kUpdTok * kPieces; i += kUpdThreads) {
    const int t = i / kPieces, p = i - t * kPieces;
    const bool ok = t < ntok && p * 8 < nch;
    cp_async16(smem_addr(x_s + t * kUpdCh * 2 + p * 16), ok ? mod.x + (b0 + t) * mod.D + c0 + p * 8 : mod.x,
               ok ? 16u : 0u);
  }
  for (int i = threadIdx.x; i < kUpdTok * kPieces * S; i += kUpdThreads) {
    const int t = i / (kPieces * S), p = i - t * kPieces * S;  // 16-byte piece p of the token's row
    const bool ok = t < ntok && p * 8 < nch * S;
    cp_async16(smem_addr(cache_s + t * kUpdCh * S * 2 + p * 16),
               ok ? mod.cache + ((b0 + t) * mod.D + c0) * S + p * 8 : mod.cache, ok ? 16u : 0u);
  }
  cp_async_commit();
  griddep_wait();  // alpha comes from the router grid
  for (int i = threadIdx.x; i < kUpdTok * kDecKP; i += kUpdThreads) {
    const int t = i / kDecKP, k = i - t * kDecKP;
    const bool ok = t < ntok && k < mod.K;
    reinterpret_cast<bf16*>(alpha_s + t * kUpdAlphaPitch)[k] = ok ? mod.alpha[(b0 + t) * mod.K + k] : bf16(0.f);
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- W_s = alpha . basis_s for the warp's 16 channels (two 8-channel n-tiles) and the
  // CTA's 16 tokens, into w_s [tap][token][64 channels] fp32
  uint32_t af[4];
  ldsm_x4(smem_addr(alpha_s) + lm_row_d(lane) * kUpdAlphaPitch + lm_col_d(lane) * 2, af);
  const int cw = warp * 16;
#pragma unroll
  for (int s = 0; s < S; ++s) {
    uint32_t bf[4];
    ldsm_x4_t(smem_addr(basis_s) + (s * kDecKP + lm_row_d(lane)) * kUpdBasisPitch + (cw + lm_col_d(lane)) * 2, bf);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float w[4];
      mma_bf16_z(w, af, bf[2 * nt], bf[2 * nt + 1]);  // w[2h + e]: token g + 8h, channel cw + 8nt + 2q + e
#pragma unroll
      for (int h = 0; h < 2; ++h)
        *reinterpret_cast<float2*>(w_s + (s * kUpdTok + g + 8 * h) * kUpdWPitch + (cw + 8 * nt + 2 * q) * 4) =
            make_float2(w[2 * h], w[2 * h + 1]);
    }
  }
  __syncthreads();

  // ---- thread = (token, channel pair): y = [silu](sum_s state_s * W_s) with state_s = cache
  // slot s+1, x for the newest tap; the pair's two cache rows shift in place, x appended
#pragma unroll
  for (int it = 0; it < kUpdTok * (kUpdCh / 2) / kUpdThreads; ++it) {
    const int item = it * kUpdThreads + threadIdx.x;
    const int t = item / (kUpdCh / 2), ch = 2 * (item - t * (kUpdCh / 2));
    const uint32_t xp = *reinterpret_cast<const uint32_t*>(x_s + (t * kUpdCh + ch) * 2);
    uint32_t cr[S];  // rows of channels ch, ch+1: S slots each, 2*S bf16
    char* crow = cache_s + (t * kUpdCh + ch) * S * 2;
#pragma unroll
    for (int i = 0; i < S; ++i) cr[i] = reinterpret_cast<const uint32_t*>(crow)[i];
    auto slot = [&](int e, int i) -> uint32_t {  // channel ch+e, slot i
      const int el = e * S + i;
      return (cr[el >> 1] >> (16 * (el & 1))) & 0xffffu;
    };
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const float2 w = *reinterpret_cast<const float2*>(w_s + (s * kUpdTok + t) * kUpdWPitch + ch * 4);
      const uint32_t s0 = s == S - 1 ? (xp & 0xffffu) : slot(0, s + 1);
      const uint32_t s1 = s == S - 1 ? (xp >> 16) : slot(1, s + 1);
      acc0 = fmaf(__uint_as_float(s0 << 16), w.x, acc0);
      acc1 = fmaf(__uint_as_float(s1 << 16), w.y, acc1);
    }
    if (mod.act) {
      acc0 = silu_f(acc0);
      acc1 = silu_f(acc1);
    }
    *reinterpret_cast<uint32_t*>(y_s + (t * kUpdCh + ch) * 2) = pack_bf16(acc0, acc1);
    uint32_t nr[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
      uint32_t half[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int el = 2 * i + j, e = el / S, sl = el - e * S;
        half[j] = sl == S - 1 ? (e == 0 ? (xp & 0xffffu) : (xp >> 16)) : slot(e, sl + 1);
      }
      nr[i] = half[0] | (half[1] << 16);
    }
#pragma unroll
    for (int i = 0; i < S; ++i) reinterpret_cast<uint32_t*>(crow)[i] = nr[i];
  }
  __syncthreads();

  // ---- stores (16-byte pieces)
  for (int i = threadIdx.x; i < kUpdTok * kPieces; i += kUpdThreads) {
    const int t = i / kPieces, p = i - t * kPieces;
    if (t < ntok && p * 8 < nch)
      *reinterpret_cast<uint4*>(mod.out + (b0 + t) * mod.D + c0 + p * 8) =
          *reinterpret_cast<const uint4*>(y_s + t * kUpdCh * 2 + p * 16);
  }
  for (int i = threadIdx.x; i < kUpdTok * kPieces * S; i += kUpdThreads) {
    const int t = i / (kPieces * S), p = i - t * kPieces * S;
    if (t < ntok && p * 8 < nch * S)
      *reinterpret_cast<uint4*>(mod.cache + ((b0 + t) * mod.D + c0) * S + p * 8) =
          *reinterpret_cast<const uint4*>(cache_s + t * kUpdCh * S * 2 + p * 16);
  }
}

int g_dec_sm_configured[64];

template <int S>
cudaError_t launch_update(dim3 grid, const DecArgs& a, cudaStream_t st, int dev) {
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(k_dec_update<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, UpdLayout<S>::total);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  // launched as a programmatic dependent of the router (its loads overlap the router)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kUpdThreads);
  cfg.dynamicSmemBytes = UpdLayout<S>::total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_dec_update<S>, a);
}

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
    case 1: e = launch_update<1>(grid, a, st, dev); break;
    case 2: e = launch_update<2>(grid, a, st, dev); break;
    case 3: e = launch_update<3>(grid, a, st, dev); break;
    case 4: e = launch_update<4>(grid, a, st, dev); break;
    default: return MOC_ERR_UNSUPPORTED_SHAPE;
  }
  if (e != cudaSuccess) return note_cuda(e);
  note_launch();
  return note_cuda(cudaGetLastError());
}

}  // namespace moc
