// Fused decode step for several MoC modules that share the routing input z (the q / k / v
// convolutions of an attention block, reference README.md:120-129), bf16.
//
// One launch for all modules instead of a router GEMM, an activation and an update kernel
// per module.  k_dec_step runs as clusters of 8 CTAs; a cluster covers 16 tokens and up to
// 8 x 128 channels of one module (a module wider than 1024 channels takes several
// clusters, each of which routes the 16 tokens itself).  Each CTA:
//   1. issues the loads of its share of the router operands: warp w of CTA r owns the
//      32-column groups r*8 + w, r*8 + w + 64, ... of z_dim and reads them straight from
//      global memory into mma.sync fragments, with no shared-memory staging; then starts the
//      16-byte copies of its update tiles (the basis slice of its 128 channels, x and the
//      cache rows of its 16 tokens), which are not needed before the router has finished;
//   2. computes its share of the 16 x K router logits (bf16 -> fp32);
//   3. adds its warps' tiles in shared memory and sends the sum to CTA 0 with st.async,
//      which completes on CTA 0's mbarrier; CTA 0 adds the 8 tiles in rank order, applies
//      softmax / exp per token over 16 lanes (moc/api.py:383-388), sends the bf16 alpha tile
//      to the other CTAs the same way (each waits on its own mbarrier) and writes alpha to
//      global memory;
//   4. per tap, one ldmatrix of the basis and two mma.sync per warp form W_s = alpha . basis_s
//      for 16 tokens x 16 channels (bf16 products exact, fp32 sums: the rounding of the
//      reference's bf16 forward, moc/kernels.py:125-130; its decode kernel rounds each
//      product to bf16 first, moc/kernels.py:466-513, a difference far inside the bf16
//      tolerance).  The epilogue works on the MMA's output fragments: each thread owns
//      (token, channel pair) positions, reads the state there, forms y = [silu](sum_s
//      state_s * W_s), shifts the pair's cache rows with x appended (moc/kernels.py:522-550),
//      and y and the cache tile leave with 16-byte stores.
#include <algorithm>
#include <climits>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_mma.cuh"
#include "moc_tma.cuh"

namespace moc {

// status word of the decode kernel (bounded-wait timeouts), read by moc_device_status()
__device__ int g_dec_status;

namespace {

constexpr int kDecTok = 16;                  // tokens per cluster (MMA M)
constexpr int kDecKP = 16;                   // bases per module, padded (MMA N = 2 x 8)
constexpr int kDecCluster = 8;               // CTAs per cluster (split of z_dim and of the channels)
constexpr int kDecThreads = 256;             // 8 warps
constexpr int kDecGroupCols = 32;            // z columns per router group (two MMA k-steps)
constexpr int kDecCh = 128;                  // channels per CTA
constexpr int kDecBasisPitch = kDecCh * 2 + 16;  // padded rows: conflict-free ldmatrix
constexpr int kDecAlphaPitch = 48;
constexpr int kDecXPitch = kDecCh * 2 + 16;      // x / y rows, padded: conflict-free pair reads

template <int S>
struct DecLayout {
  static constexpr int cache_pitch = kDecCh * S * 2 + 64;  // padded: two token rows per quarter-warp on distinct banks
  static constexpr int basis = S * kDecKP * kDecBasisPitch;
  static constexpr int alpha = kDecTok * kDecAlphaPitch;
  static constexpr int x = kDecTok * kDecXPitch;
  static constexpr int cache = kDecTok * cache_pitch;
  static constexpr int red = 8 * kDecTok * kDecKP * 4;            // per-warp logit tiles
  static constexpr int part = kDecCluster * kDecTok * kDecKP * 4;  // CTA 0: the cluster's CTA sums
  static constexpr int bars = 16;                                  // two mbarriers
  static constexpr int total = basis + alpha + x + cache + red + part + bars;
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
  int n_parts;  // clusters per 16-token group, over all modules
  int64_t B, Dz;
  const bf16* z;
  int part_prefix[MOC_DECODE_MAX_MODULES + 1];  // clusters per token group, prefix sums over modules
};

__device__ __forceinline__ int lm_row_d(int lane) { return (lane & 7) + ((lane >> 3) & 1) * 8; }
__device__ __forceinline__ int lm_col_d(int lane) { return (lane >> 4) * 8; }

// Both cluster barriers of the kernel are split into an arrive and a wait.  The first: arrive
// at the start (after the mbarrier initialisation), wait before the first store into another
// CTA's shared memory, so that every CTA of the cluster is running with its mbarriers ready.
// The second: arrive after the CTA's last store into another CTA, wait just before exit, so
// that no CTA leaves while another may still write into its shared memory.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

// Address of the shared-memory location `addr` (this CTA's layout) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(addr), "r"(rank));
  return remote;
}
// Asynchronous 4-byte store into another CTA's shared memory; its arrival counts 4 bytes
// on that CTA's mbarrier (`remote_bar`, mapped like `remote_addr`).
__device__ __forceinline__ void st_async_b32(uint32_t remote_addr, uint32_t remote_bar, uint32_t v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];\n" ::"r"(remote_addr),
               "r"(v), "r"(remote_bar)
               : "memory");
}
// Polls this CTA's mbarrier phase `parity` at most kSpinLimit times, with acquire at cluster
// scope (the bytes it counts were written by other CTAs); true once the phase completed.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, uint32_t limit = kSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ uint4 ldg16_or_zero(const bf16* p, bool ok) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (ok) v = __ldg(reinterpret_cast<const uint4*>(p));
  return v;
}

template <int S>
__global__ void __cluster_dims__(kDecCluster, 1, 1) __launch_bounds__(kDecThreads, 3)
    k_dec_step(const __grid_constant__ DecArgs a) {
  extern __shared__ __align__(128) char smem[];
  using L = DecLayout<S>;
  char* basis_s = smem;                // [tap][base][128 ch], bases past K zero
  char* alpha_s = basis_s + L::basis;  // [token][16 bases]
  char* x_s = alpha_s + L::alpha;      // [token][128 ch]; y replaces x in place
  char* cache_s = x_s + L::x;          // [token][128 ch][S]
  float* red = reinterpret_cast<float*>(cache_s + L::cache);  // [8 warps][16 tokens][16 bases]
  float* part = red + 8 * kDecTok * kDecKP;                    // [8 ranks][16 tokens][16 bases]
  const int cid = static_cast<int>(blockIdx.x / kDecCluster);
  const int tg = cid / a.n_parts, cl = cid - tg * a.n_parts;  // token group, cluster within it
  int m = 0;
  while (m + 1 < a.n_mod && cl >= a.part_prefix[m + 1]) ++m;
  const DecModule& mod = a.m[m];
  const int part_idx = cl - a.part_prefix[m];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t rank = cluster_rank();
  const int64_t b0 = static_cast<int64_t>(tg) * kDecTok;
  const int64_t c0 = (static_cast<int64_t>(part_idx) * kDecCluster + rank) * kDecCh;
  const bool has_blk = c0 < mod.D;  // CTA-uniform
  const int nch = has_blk ? static_cast<int>(mod.D - c0 < kDecCh ? mod.D - c0 : kDecCh) : 0;  // multiple of 8
  const int ntok = static_cast<int>(a.B - b0 < kDecTok ? a.B - b0 : kDecTok);
  const uint32_t bar_part = smem_addr(reinterpret_cast<char*>(part) + L::part);  // CTA 0: the other CTAs' tiles
  const uint32_t bar_alpha = bar_part + 8;                                         // CTAs 1..7: the alpha tile
  if (threadIdx.x == 0) {
    mbar_init(bar_part, 1);
    mbar_init(bar_alpha, 1);
    if (rank == 0)
      mbar_expect_tx(bar_part, (kDecCluster - 1) * kDecTok * kDecKP * 4);
    else
      mbar_expect_tx(bar_alpha, kDecTok * kDecKP * 2);
    fence_mbar_init();
  }
  cluster_arrive_relaxed();

  // ---- 1. router loads of the first pair of column groups, then the copies of the update
  // tiles, which are not needed before the router has finished.
  // Router: lane (g, q) reads columns 8q..8q+7 of a 32-column group for tokens g, g+8 and
  // bases g, g+8 (one 16-byte load each); the MMA k-slots 2q, 2q+1, 2q+8, 2q+9 of the first
  // k-step take columns 8q..8q+3, those of the second 8q+4..8q+7 (A and B use the same
  // order, and a dot product does not depend on it).  Warp w of CTA r owns the groups
  // r*8 + w, r*8 + w + 64, ...
  const int n_groups = static_cast<int>((a.Dz + kDecGroupCols - 1) / kDecGroupCols);
  const bool ok_lo = b0 + g < a.B, ok_hi = b0 + g + 8 < a.B;
  const bool ok_w0 = g < mod.K, ok_w1 = g + 8 < mod.K;
  const bf16* z_lo = a.z + (ok_lo ? b0 + g : 0) * a.Dz;
  const bf16* z_hi = a.z + (ok_hi ? b0 + g + 8 : 0) * a.Dz;
  const bf16* w0 = mod.w + static_cast<int64_t>(ok_w0 ? g : 0) * a.Dz;
  const bf16* w1 = mod.w + static_cast<int64_t>(ok_w1 ? g + 8 : 0) * a.Dz;
  constexpr int kStride = kDecCluster * 8;  // groups per sweep of the cluster's 64 warps
  uint4 v[2][4];  // [group of the pair][z token g, z token g+8, w base g, w base g+8]
  auto load_pair = [&](int gi) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int gu = gi + u * kStride;
      const int64_t col = static_cast<int64_t>(gu) * kDecGroupCols + 8 * q;
      const bool okc = gu < n_groups && col < a.Dz;  // z_dim is a multiple of 8
      v[u][0] = ldg16_or_zero(z_lo + col, okc && ok_lo);
      v[u][1] = ldg16_or_zero(z_hi + col, okc && ok_hi);
      v[u][2] = ldg16_or_zero(w0 + col, okc && ok_w0);
      v[u][3] = ldg16_or_zero(w1 + col, okc && ok_w1);
    }
  };
  int gi = static_cast<int>(rank) * 8 + warp;
  load_pair(gi);

  // update tiles (16-byte pieces; missing channels, tokens and bases become zeros)
  constexpr int kPieces = kDecCh / 8;  // 16-byte pieces per 128-channel row
  if (has_blk) {
    for (int i = threadIdx.x; i < S * kDecKP * kPieces; i += kDecThreads) {
      const int row = i / kPieces, p = i - row * kPieces;  // row = s * 16 + k
      const int s = row / kDecKP, k = row - s * kDecKP;
      const bool ok = k < mod.K && p * 8 < nch;
      cp_async16(smem_addr(basis_s + row * kDecBasisPitch + p * 16),
                 ok ? mod.basis + (static_cast<int64_t>(k) * S + s) * mod.D + c0 + p * 8 : mod.basis,
                 ok ? 16u : 0u);
    }
    for (int i = threadIdx.x; i < kDecTok * kPieces; i += kDecThreads) {
      const int t = i / kPieces, p = i - t * kPieces;
      const bool ok = t < ntok && p * 8 < nch;
      cp_async16(smem_addr(x_s + t * kDecXPitch + p * 16), ok ? mod.x + (b0 + t) * mod.D + c0 + p * 8 : mod.x,
                 ok ? 16u : 0u);
    }
    for (int i = threadIdx.x; i < kDecTok * kPieces * S; i += kDecThreads) {
      const int t = i / (kPieces * S), p = i - t * kPieces * S;  // 16-byte piece p of the token's row
      const bool ok = t < ntok && p * 8 < nch * S;
      cp_async16(smem_addr(cache_s + t * L::cache_pitch + p * 16),
                 ok ? mod.cache + ((b0 + t) * mod.D + c0) * S + p * 8 : mod.cache, ok ? 16u : 0u);
    }
    cp_async_commit();
  }

  // ---- 2. router logits of this CTA's column groups
  float acc[2][4] = {};
#pragma unroll 1
  for (;;) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t a_lo[4] = {v[u][0].x, v[u][1].x, v[u][0].y, v[u][1].y};
      const uint32_t a_hi[4] = {v[u][0].z, v[u][1].z, v[u][0].w, v[u][1].w};
      mma_bf16(acc[0], a_lo, v[u][2].x, v[u][2].y);
      mma_bf16(acc[1], a_lo, v[u][3].x, v[u][3].y);
      mma_bf16(acc[0], a_hi, v[u][2].z, v[u][2].w);
      mma_bf16(acc[1], a_hi, v[u][3].z, v[u][3].w);
    }
    gi += 2 * kStride;
    if (gi >= n_groups) break;
    load_pair(gi);
  }

  // ---- 3. reduction: warps in shared memory, CTAs in CTA 0's shared memory, in rank order.
  // acc[nt][2h + e] = partial logit (token g + 8h, base 8nt + 2q + e) of this warp's columns
  {
    float* r = red + warp * kDecTok * kDecKP;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        *reinterpret_cast<float2*>(r + (g + 8 * h) * kDecKP + nt * 8 + 2 * q) =
            make_float2(acc[nt][2 * h], acc[nt][2 * h + 1]);
  }
  __syncthreads();
  const int t = threadIdx.x >> 4, k = threadIdx.x & 15;  // 16 lanes per token
  float l = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) l += red[w * kDecTok * kDecKP + t * kDecKP + k];
  const uint32_t part_off = smem_addr(part + (rank * kDecTok + t) * kDecKP + k);
  cluster_wait();  // every CTA of the cluster is running, its mbarriers initialised
  bool timed_out;
  if (rank != 0) {
    st_async_b32(map_rank(part_off, 0), map_rank(bar_part, 0), __float_as_uint(l));
    cluster_arrive_relaxed();  // this CTA's last store into another CTA
    timed_out = !mbar_wait_cluster(bar_alpha, 0);
  } else {
    part[t * kDecKP + k] = l;
    timed_out = !mbar_wait_cluster(bar_part, 0);
    __syncthreads();  // this CTA's own tile, written above
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
    const bool ok = t < ntok && k < mod.K;  // padding tokens and bases get alpha 0
    const bf16 vb = __float2bfloat16_rn(ok ? v : 0.f);
    const uint32_t bits = __bfloat16_as_ushort(vb);
    const uint32_t hi = __shfl_down_sync(0xffffffffu, bits, 1);  // base k + 1 of the same token
    if ((k & 1) == 0) {  // one 4-byte store per base pair
      const uint32_t pair = bits | (hi << 16);
      const uint32_t off = smem_addr(alpha_s + t * kDecAlphaPitch + k * 2);
      *reinterpret_cast<uint32_t*>(alpha_s + t * kDecAlphaPitch + k * 2) = pair;
#pragma unroll
      for (int rr = 1; rr < kDecCluster; ++rr) st_async_b32(map_rank(off, rr), map_rank(bar_alpha, rr), pair);
    }
    cluster_arrive_relaxed();  // this CTA's last store into another CTA
    if (ok && part_idx == 0) mod.alpha[(b0 + t) * mod.K + k] = vb;
  }
  timed_out = __syncthreads_or(timed_out);  // also: CTA 0's alpha tile is complete
  if (timed_out) {
    if (threadIdx.x == 0) atomicOr(&g_dec_status, kStatusWaitTimeout);
    mbar_wait_cluster(rank == 0 ? bar_part : bar_alpha, 0);  // once more, bounded: stores still on the way
  }

  // ---- 4. update
  cp_async_wait<0>();
  if (has_blk && !timed_out) {
    __syncthreads();
    uint32_t af[4];
    ldsm_x4(smem_addr(alpha_s) + lm_row_d(lane) * kDecAlphaPitch + lm_col_d(lane) * 2, af);
    const int cw = warp * 16;
    // this thread's outputs: tokens g + 8h, channels cw + 8nt + 2q + e (the MMA's C fragment)
    uint32_t cr[2][2][S];  // [h][nt]: cache rows of the channel pair, S slots each, 2*S bf16
    uint32_t xp[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int tt = g + 8 * h, c = cw + 8 * nt + 2 * q;
        const uint32_t* row = reinterpret_cast<const uint32_t*>(cache_s + tt * L::cache_pitch + c * S * 2);
#pragma unroll
        for (int i = 0; i < S; ++i) cr[h][nt][i] = row[i];
        xp[h][nt] = *reinterpret_cast<const uint32_t*>(x_s + tt * kDecXPitch + c * 2);
      }
    auto slot = [&](int h, int nt, int e, int i) -> uint32_t {  // channel c+e, slot i
      const int el = e * S + i;
      return (cr[h][nt][el >> 1] >> (16 * (el & 1))) & 0xffffu;
    };
    float y[2][4] = {};  // [nt][2h + e]
#pragma unroll
    for (int s = 0; s < S; ++s) {
      uint32_t bf[4];
      ldsm_x4_t(smem_addr(basis_s) + (s * kDecKP + lm_row_d(lane)) * kDecBasisPitch + (cw + lm_col_d(lane)) * 2, bf);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float w[4];
        mma_bf16_z(w, af, bf[2 * nt], bf[2 * nt + 1]);  // w[2h + e]: token g + 8h, channel cw + 8nt + 2q + e
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            // state_s = cache slot s+1; x for the newest tap
            const uint32_t st = s == S - 1 ? ((xp[h][nt] >> (16 * e)) & 0xffffu) : slot(h, nt, e, s + 1);
            y[nt][2 * h + e] = fmaf(__uint_as_float(st << 16), w[2 * h + e], y[nt][2 * h + e]);
          }
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int tt = g + 8 * h, c = cw + 8 * nt + 2 * q;
        float y0 = y[nt][2 * h], y1 = y[nt][2 * h + 1];
        if (mod.act) {
          y0 = silu_f(y0);
          y1 = silu_f(y1);
        }
        *reinterpret_cast<uint32_t*>(x_s + tt * kDecXPitch + c * 2) = pack_bf16(y0, y1);
        uint32_t* row = reinterpret_cast<uint32_t*>(cache_s + tt * L::cache_pitch + c * S * 2);
#pragma unroll
        for (int i = 0; i < S; ++i) {
          uint32_t half[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int el = 2 * i + j, e = el / S, sl = el - e * S;
            half[j] = sl == S - 1 ? ((xp[h][nt] >> (16 * e)) & 0xffffu) : slot(h, nt, e, sl + 1);
          }
          row[i] = half[0] | (half[1] << 16);
        }
      }
    __syncthreads();

    // ---- stores (16-byte pieces)
    for (int i = threadIdx.x; i < kDecTok * kPieces; i += kDecThreads) {
      const int tt = i / kPieces, p = i - tt * kPieces;
      if (tt < ntok && p * 8 < nch)
        *reinterpret_cast<uint4*>(mod.out + (b0 + tt) * mod.D + c0 + p * 8) =
            *reinterpret_cast<const uint4*>(x_s + tt * kDecXPitch + p * 16);
    }
    for (int i = threadIdx.x; i < kDecTok * kPieces * S; i += kDecThreads) {
      const int tt = i / (kPieces * S), p = i - tt * kPieces * S;
      if (tt < ntok && p * 8 < nch * S)
        *reinterpret_cast<uint4*>(mod.cache + ((b0 + tt) * mod.D + c0) * S + p * 8) =
            *reinterpret_cast<const uint4*>(cache_s + tt * L::cache_pitch + p * 16);
    }
  }
  cluster_wait();  // no CTA of the cluster still stores into this one
}

// The decode step's cross-CTA wait with nothing to wait for: CTA 1 of the pair sends no
// bytes, so CTA 0's wait runs out of polls and records the timeout; both CTAs then leave
// through the exit barrier, as k_dec_step does.
__global__ void __cluster_dims__(2, 1, 1) k_dec_wait_probe(uint32_t limit) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    mbar_expect_tx(b, 4);
    fence_mbar_init();
  }
  cluster_arrive_relaxed();
  cluster_wait();
  bool ok = true;
  if (cluster_rank() == 0) ok = mbar_wait_cluster(b, 0, limit);
  if (!ok && threadIdx.x == 0) atomicOr(&g_dec_status, kStatusWaitTimeout);
  cluster_arrive_relaxed();
  cluster_wait();
}

template <int S>
cudaError_t launch_step(unsigned grid, const DecArgs& a, cudaStream_t st, int dev) {
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(k_dec_step<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecLayout<S>::total);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  k_dec_step<S><<<grid, kDecThreads, DecLayout<S>::total, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

int decode_step_multi(int n, const moc_decode_module* mods, int64_t B, int64_t Dz, const void* z, cudaStream_t st) {
  DecArgs a{};
  a.n_mod = n;
  a.B = B;
  a.Dz = Dz;
  a.z = static_cast<const bf16*>(z);
  const int S = mods[0].kernel_size;
  a.part_prefix[0] = 0;
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
    a.part_prefix[i + 1] = a.part_prefix[i] + static_cast<int>(ceil_div(ceil_div(m.D, kDecCh), kDecCluster));
  }
  a.n_parts = a.part_prefix[n];
  if (B == 0) return MOC_OK;
  const int64_t ctas = ceil_div(B, kDecTok) * a.n_parts * kDecCluster;
  if (ctas > INT_MAX) return MOC_ERR_UNSUPPORTED_SHAPE;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return note_cuda(e);
  const unsigned grid = static_cast<unsigned>(ctas);
  switch (S) {
    case 1: e = launch_step<1>(grid, a, st, dev); break;
    case 2: e = launch_step<2>(grid, a, st, dev); break;
    case 3: e = launch_step<3>(grid, a, st, dev); break;
    case 4: e = launch_step<4>(grid, a, st, dev); break;
    default: return MOC_ERR_UNSUPPORTED_SHAPE;
  }
  if (e != cudaSuccess) return note_cuda(e);
  note_launch();
  return MOC_OK;
}

int decode_wait_timeout_probe(uint32_t limit, cudaStream_t st) {
  k_dec_wait_probe<<<2, 32, 0, st>>>(limit);
  note_launch();
  return note_cuda(cudaGetLastError());
}

int decode_status(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_dec_status, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_dec_status, &zero, sizeof(int));
    if (e != cudaSuccess) return note_cuda(e);
  }
  *out = v;
  return MOC_OK;
}

}  // namespace moc
