// Tensor-core router for bf16: alpha = softmax/exp(z @ W^T) and its backward.
//
// Replaces the reference's F.linear + torch.softmax / torch.exp and their autograd
// (moc/api.py:383-388).  The projection [N, Dz] x [Dz, K] is tall and skinny (K <= 32),
// so both kernels are bound by streaming z (and writing dz) through HBM:
//
//   forward : a CTA owns 64 token rows and streams their z rows in 128-column chunks
//             through a 4-stage cp.async ring; each warp accumulates a 16 x K logit tile
//             with mma.sync (fp32) and applies softmax (over the 4 lanes of a quad that
//             hold one row) or exp before writing alpha.  Logits never leave registers.
//   backward: dlogits = alpha*(dalpha - sum alpha*dalpha) (softmax) or alpha*dalpha (exp),
//             then dz = dlogits @ W and dW = dlogits^T @ z in one pass over z: a CTA owns a
//             128-column slice of Dz and a contiguous token range, writes its dz columns and
//             keeps dW^T for its slice in registers; a second kernel adds the per-CTA dW
//             partials in a fixed order (deterministic).
#include <algorithm>
#include <mutex>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_mma.cuh"
#include "moc_tma.cuh"

namespace moc {
namespace {

constexpr int kZC = 128;             // z columns per chunk / slice
constexpr int kRowB = (kZC + 8) * 2; // 272 B smem row
constexpr int kFwdRows = 64;         // tokens per forward CTA
constexpr int kFwdStages = 4;
constexpr int kBwdTile = 64;         // tokens per backward tile

__device__ __forceinline__ int lm_row(int lane) { return (lane & 7) + ((lane >> 3) & 1) * 8; }
__device__ __forceinline__ int lm_col(int lane) { return (lane >> 4) * 8; }

// ------------------------------------------------------------------ forward

__device__ int g_router_status;  // kStatus* bits of bounded waits that ran out

template <int KT>
struct FwdLayout {
  static constexpr int KP = KT * 16;
  static constexpr int zbox = kFwdRows * 128;  // one 64-token x 64-column box, 128 B rows
  static constexpr int wbox = KP * 128;        // one KP-base x 64-column box
  static constexpr int stage_bytes = 2 * zbox + 2 * wbox;  // 128 columns of z and W
  static constexpr int tx_bytes = stage_bytes;
  static constexpr int total = kFwdStages * stage_bytes + 1024 + 64;  // + alignment slack + mbarriers
};

// TMA-staged forward: thread 0 keeps kFwdStages chunks of 128 z columns (two 64-column
// boxes of z and of W, 128-byte swizzled) in flight on per-stage mbarriers.
template <int KT>
__global__ void __launch_bounds__(128) k_router_fwd_tc(const __grid_constant__ CUtensorMap zmap,
                                                       const __grid_constant__ CUtensorMap wmap,
                                                       bf16* __restrict__ alpha, int64_t N, int64_t Dz, int K,
                                                       int act) {
  using L = FwdLayout<KT>;
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + kFwdStages * L::stage_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kFwdRows;
  const int n_chunks = static_cast<int>((Dz + kZC - 1) / kZC);

  auto issue = [&](int c) {
    const int st = c % kFwdStages;
    const uint32_t dst = sbase + st * L::stage_bytes;
    const uint32_t bar = bar0 + 8 * st;
    mbar_expect_tx(bar, L::tx_bytes);
    tma_load_2d(dst, &zmap, c * kZC, static_cast<int>(t0), bar);
    tma_load_2d(dst + L::zbox, &zmap, c * kZC + 64, static_cast<int>(t0), bar);
    tma_load_2d(dst + 2 * L::zbox, &wmap, c * kZC, 0, bar);
    tma_load_2d(dst + 2 * L::zbox + L::wbox, &wmap, c * kZC + 64, 0, bar);
  };

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&zmap);
    tma_prefetch_desc(&wmap);
    for (int st = 0; st < kFwdStages; ++st) mbar_init(bar0 + 8 * st, 1);
    fence_mbar_init();
  }
  griddep_wait();  // z may come from the kernels before this one
  __syncthreads();
  if (threadIdx.x == 0)
    for (int c = 0; c < kFwdStages && c < n_chunks; ++c) issue(c);

  float acc[2 * KT][4] = {};
  for (int c = 0; c < n_chunks; ++c) {
    const int st = c % kFwdStages;
    const bool ok = mbar_wait(bar0 + 8 * st, (c / kFwdStages) & 1);
    if (__syncthreads_or(!ok)) {
      // a copy did not land in time: record it, wait (bounded) for what is in flight, stop
      if (threadIdx.x == 0) {
        atomicOr(&g_router_status, kStatusWaitTimeout);
        for (int cc = c; cc < n_chunks && cc < c + kFwdStages; ++cc)
          mbar_wait(bar0 + 8 * (cc % kFwdStages), (cc / kFwdStages) & 1);
      }
      return;
    }
    const uint32_t zs = sbase + st * L::stage_bytes;
    const uint32_t ws = zs + 2 * L::zbox;
#pragma unroll
    for (int kk = 0; kk < kZC / 16; ++kk) {
      uint32_t af[4];
      {
        const int row = warp * 16 + lm_row(lane);
        const int c16 = kk * 2 + (lane >> 4);
        ldsm_x4(zs + (c16 >> 3) * L::zbox + sw128(row, c16 & 7), af);
      }
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        uint32_t bb[4];  // (k 0-7 | 8-15) x (z columns 0-7 | 8-15) of this 16-base group
        const int k = kt * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c16 = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(ws + (c16 >> 3) * L::wbox + sw128(k, c16 & 7), bb);
        mma_bf16(acc[2 * kt], af, bb[0], bb[1]);
        mma_bf16(acc[2 * kt + 1], af, bb[2], bb[3]);
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
    if (threadIdx.x == 0 && c + kFwdStages < n_chunks) issue(c + kFwdStages);
  }
  griddep_launch_dependents();  // only the epilogue is left

  // acc[kn][2h + e] = logit(token warp*16 + g + 8h, base 8kn + 2q + e); the 4 lanes of a
  // quad hold one token row.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = -INFINITY;
    if (act == 0) {
#pragma unroll
      for (int kn = 0; kn < 2 * KT; ++kn)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (kn * 8 + 2 * q + e < K) mx = fmaxf(mx, acc[kn][2 * h + e]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    } else {
      mx = 0.f;
    }
    float ev[2 * KT][2];
    float sum = 0.f;
#pragma unroll
    for (int kn = 0; kn < 2 * KT; ++kn)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        ev[kn][e] = kn * 8 + 2 * q + e < K ? expf(acc[kn][2 * h + e] - mx) : 0.f;
        sum += ev[kn][e];
      }
    float inv = 1.f;
    if (act == 0) {
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      inv = 1.f / sum;
    }
    const int64_t tok = t0 + warp * 16 + g + 8 * h;
    if (tok < N) {
#pragma unroll
      for (int kn = 0; kn < 2 * KT; ++kn) {
        const int k = kn * 8 + 2 * q;
        if (k < K)
          *reinterpret_cast<uint32_t*>(alpha + tok * K + k) = pack_bf16(ev[kn][0] * inv, ev[kn][1] * inv);
      }
    }
  }
}

// Diagnostic: waits on an mbarrier that nothing arrives on, with `limit` polls, and
// records the timeout exactly like the staging kernels do.
__global__ void k_wait_timeout_probe(uint32_t limit) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_addr(&bar);
  mbar_init(b, 1);
  fence_mbar_init();
  if (!mbar_wait(b, 0, limit)) atomicOr(&g_router_status, kStatusWaitTimeout);
}

// ------------------------------------------------------------------ backward

template <int KT>
struct BwdLayout {
  static constexpr int KP = KT * 16;
  static constexpr int DLB = (KP + 8) * 2;       // dl row bytes (padded, conflict-free ldmatrix)
  static constexpr int zbox = kBwdTile * 128;    // one 64-token x 64-column box, 128 B rows (swizzled)
  static constexpr int z_bytes = 2 * zbox;       // 128 columns
  static constexpr int w_bytes = KP * kRowB;
  static constexpr int dl_bytes = kBwdTile * DLB;  // one of two dl buffers
  static constexpr int ost_bytes = 8 * 16 * 32;   // per-warp dz staging: 16 rows x 16 columns bf16
  static constexpr int total = 1024 + 2 * z_bytes + w_bytes + 2 * dl_bytes + ost_bytes + 64;
};

struct RouterBwdArgs {
  const bf16* w;
  const bf16* alpha;
  const void* dalpha;
  int da_dtype;
  bf16* dz;
  float* dw_part;  // [groups][K][Dz]
  int64_t N, Dz;
  int K, act;
  int64_t tiles_per_group;
  int vec_ad;  // alpha and dalpha bf16 and 16-byte aligned: vector loads of a thread's bases
  int vec_dz;  // dz 16-byte aligned: 16-byte stores of staged rows
};

// TMA-staged backward: thread 0 double-buffers 64-token x 128-column z tiles (two
// 128B-swizzled boxes) on mbarriers; every thread computes dlogits for the next tile's
// tokens meanwhile.  At most 72 registers for two base groups: three CTAs per SM, so that the
// grid (sized for 3 per SM) is one wave.
template <int KT>
__global__ void __launch_bounds__(256, (KT == 1 ? 4 : 3)) k_router_bwd_tc(const __grid_constant__ CUtensorMap zmap,
                                                      const __grid_constant__ CUtensorMap dzmap, RouterBwdArgs a) {
  using L = BwdLayout<KT>;
  constexpr int KP = L::KP;
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t z_st = smem_addr(smem);
  char* w_s = smem + 2 * L::z_bytes;
  char* dl_s = w_s + L::w_bytes;
  char* ost = dl_s + 2 * L::dl_bytes;
  const uint32_t bar0 = smem_addr(ost + L::ost_bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t col_base = static_cast<int64_t>(blockIdx.x) * kZC;
  const int64_t n_tiles = (a.N + kBwdTile - 1) / kBwdTile;
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * a.tiles_per_group;
  const int64_t i1 = i0 + a.tiles_per_group < n_tiles ? i0 + a.tiles_per_group : n_tiles;
  const int cw = warp * 16;  // this warp's 16 columns inside the slice
  const bool want_dz = a.dz != nullptr;
  const bool want_dw = a.dw_part != nullptr;
  // zT ldmatrix: rows (lane&7) + (lane>>4)*8, 16-byte chunk 2*(warp&3) + ((lane>>3)&1) of box warp>>2
  const uint32_t zt_box = static_cast<uint32_t>((warp >> 2) * L::zbox);
  const int zt_row = (lane & 7) + (lane >> 4) * 8;
  const int zt_chunk = 2 * (warp & 3) + ((lane >> 3) & 1);

  auto issue = [&](int64_t tile, int stage) {
    const uint32_t bar = bar0 + 8 * stage;
    const uint32_t dst = z_st + stage * L::z_bytes;
    fence_proxy_async();
    mbar_expect_tx(bar, L::z_bytes);
    tma_load_2d(dst, &zmap, static_cast<int>(col_base), static_cast<int>(tile * kBwdTile), bar);
    tma_load_2d(dst + L::zbox, &zmap, static_cast<int>(col_base) + 64, static_cast<int>(tile * kBwdTile), bar);
  };

  float dwa[2 * KT][4] = {};  // dW^T: (column cw + g | +8) x (base 8kn + 2q..)
  uint32_t wb[KT][4];         // W as the B operand of dz = dl . W (this warp's 16 columns)
  if (i0 < i1) {
    if (threadIdx.x == 0) {
      tma_prefetch_desc(&zmap);
      mbar_init(bar0, 1);
      mbar_init(bar0 + 8, 1);
      fence_mbar_init();
    }
    for (int idx = threadIdx.x; idx < KP * 16; idx += 256) {
      const int k = idx >> 4, chunk = idx & 15;
      const int64_t col = col_base + chunk * 8;
      const bool ok = k < a.K && col < a.Dz;
      cp_async16(smem_addr(w_s + k * kRowB + chunk * 16), ok ? a.w + k * a.Dz + col : a.w, ok ? 16u : 0u);
    }
    cp_async_commit();
    griddep_wait();  // z, alpha and dalpha may come from the kernels before this one
    __syncthreads();
    if (threadIdx.x == 0) issue(i0, 0);
    cp_async_wait<0>();
    __syncthreads();
#pragma unroll
    for (int kt = 0; kt < KT; ++kt)
      ldsm_x4_t(smem_addr(w_s + (kt * 16 + lm_row(lane)) * kRowB + (cw + lm_col(lane)) * 2), wb[kt]);
  }
  if (i0 >= i1) griddep_wait();  // a CTA without tiles still writes its (zero) dW partial
  // alpha / dalpha of the next tile are loaded one iteration ahead into registers: four
  // threads per token, each owning KP/4 bases.  The bf16 pairs stay packed until the next
  // iteration uses them, so nothing waits on the loads before then.
  constexpr int KQ = KP / 4;
  const int dl_row = threadIdx.x >> 2, dl_part = threadIdx.x & 3;
  float av[KQ], dv[KQ];               // the element path: values
  uint32_t wa[KQ / 2], wd[KQ / 2];    // the vector path: packed bf16 pairs
  auto fetch = [&](int64_t tile) {
    const int64_t tok = tile * kBwdTile + dl_row;
    if (a.vec_ad) {  // K % 8 == 0: a thread's KQ bases are all valid or all padding
#pragma unroll
      for (int e = 0; e < KQ / 2; ++e) wa[e] = 0u, wd[e] = 0u;
      if (tok < a.N && dl_part * KQ < a.K) {
        const bf16* pa = a.alpha + tok * a.K + dl_part * KQ;
        const bf16* pd = static_cast<const bf16*>(a.dalpha) + tok * a.K + dl_part * KQ;
        if constexpr (KQ == 4) {
          const uint2 va = __ldg(reinterpret_cast<const uint2*>(pa)), vd = __ldg(reinterpret_cast<const uint2*>(pd));
          wa[0] = va.x, wa[1] = va.y, wd[0] = vd.x, wd[1] = vd.y;
        } else {
#pragma unroll
          for (int v = 0; v < KQ / 8; ++v) {
            const uint4 va = __ldg(reinterpret_cast<const uint4*>(pa) + v);
            const uint4 vd = __ldg(reinterpret_cast<const uint4*>(pd) + v);
            wa[4 * v] = va.x, wa[4 * v + 1] = va.y, wa[4 * v + 2] = va.z, wa[4 * v + 3] = va.w;
            wd[4 * v] = vd.x, wd[4 * v + 1] = vd.y, wd[4 * v + 2] = vd.z, wd[4 * v + 3] = vd.w;
          }
        }
      }
      return;
    }
#pragma unroll
    for (int e = 0; e < KQ; ++e) {
      const int k = dl_part * KQ + e;
      const bool ok = tok < a.N && k < a.K;
      av[e] = ok ? __bfloat162float(a.alpha[tok * a.K + k]) : 0.f;
      dv[e] = ok ? ld_any(a.dalpha, a.da_dtype, tok * a.K + k) : 0.f;
    }
  };
  if (i0 < i1) fetch(i0);

  for (int64_t it = i0; it < i1; ++it) {
    const int cur = static_cast<int>((it - i0) & 1);
    const uint32_t parity = static_cast<uint32_t>(((it - i0) >> 1) & 1);
    char* dl_cur = dl_s + cur * L::dl_bytes;  // tile it-2 used it; its readers passed the last wait barrier
    // dlogits for this tile's 64 tokens (bf16, like the reference's bf16 autograd); the
    // softmax dot is a quad reduction.
    {
      if (a.vec_ad) {
#pragma unroll
        for (int e = 0; e < KQ / 2; ++e) {
          av[2 * e] = bf_lo(wa[e]), av[2 * e + 1] = bf_hi(wa[e]);
          dv[2 * e] = bf_lo(wd[e]), dv[2 * e + 1] = bf_hi(wd[e]);
        }
      }
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < KQ; ++e) dot = fmaf(av[e], dv[e], dot);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      if (a.act != 0) dot = 0.f;
      uint32_t o[KQ / 2];
#pragma unroll
      for (int e = 0; e < KQ / 2; ++e) o[e] = pack_bf16(av[2 * e] * (dv[2 * e] - dot), av[2 * e + 1] * (dv[2 * e + 1] - dot));
      char* dst = dl_cur + dl_row * L::DLB + dl_part * KQ * 2;  // 8-byte (KQ 4) / 16-byte (KQ 8) aligned
      if constexpr (KQ == 4) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(o[0], o[1]);
      } else {
#pragma unroll
        for (int v = 0; v < KQ / 8; ++v)
          *reinterpret_cast<uint4*>(dst + 16 * v) = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
      }
    }
    if (it + 1 < i1) fetch(it + 1);
    const bool landed = mbar_wait(bar0 + 8 * cur, parity);
    if (__syncthreads_or(!landed)) {
      if (threadIdx.x == 0) {
        atomicOr(&g_router_status, kStatusWaitTimeout);
        mbar_wait(bar0 + 8 * cur, parity);
        bulk_wait<0>();
      }
      // this CTA's dW partial is incomplete: it is written as NaN, so the reduction of the
      // partials (which reads every group) cannot return a finite mix of this call's and
      // an earlier call's values
      if (want_dw) {
        for (int kn = 0; kn < 2 * KT; ++kn)
          for (int e = 0; e < 4; ++e) dwa[kn][e] = __int_as_float(0x7fc00000);
        break;
      }
      return;
    }
    // every thread is past tile it-1, so its stage can be refilled with tile it+1 once the
    // dz store of tile it-1 has read it
    if (threadIdx.x == 0 && it + 1 < i1) {
      bulk_wait_read<0>();
      issue(it + 1, cur ^ 1);
    }
    const uint32_t z_s = z_st + cur * L::z_bytes;
    const int64_t tok0 = it * kBwdTile;
    // dz of a whole tile leaves through the stage: block b's dz overwrites its z rows (this
    // warp's columns) once the block's dW products have read them, and one TMA store per box
    // writes the tile.  A partial last tile stores through the warp's staging rows.
    const bool dz_tma = want_dz && a.vec_dz && tok0 + kBwdTile <= a.N;  // uniform across the CTA
    for (int b = 0; b < kBwdTile / 16; ++b) {
      if (tok0 + 16 * b >= a.N) break;
      uint32_t af[KT][4];  // dl rows of this block (A operand of dz)
#pragma unroll
      for (int kt = 0; kt < KT; ++kt)
        ldsm_x4(smem_addr(dl_cur + (16 * b + lm_row(lane)) * L::DLB + (kt * 16 + lm_col(lane)) * 2), af[kt]);
      uint32_t dzp[4];  // this block's dz (stmatrix order) when the tile leaves by TMA
      if (want_dz) {
        // dz[tok, col] = sum_k dl[tok, k] W[k, col]
        float acc[2][4];
        mma_bf16_z(acc[0], af[0], wb[0][0], wb[0][1]);
        mma_bf16_z(acc[1], af[0], wb[0][2], wb[0][3]);
#pragma unroll
        for (int kt = 1; kt < KT; ++kt) {
          mma_bf16(acc[0], af[kt], wb[kt][0], wb[kt][1]);
          mma_bf16(acc[1], af[kt], wb[kt][2], wb[kt][3]);
        }
        if (dz_tma) {
          dzp[0] = pack_bf16(acc[0][0], acc[0][1]), dzp[1] = pack_bf16(acc[0][2], acc[0][3]);
          dzp[2] = pack_bf16(acc[1][0], acc[1][1]), dzp[3] = pack_bf16(acc[1][2], acc[1][3]);
        } else if (a.vec_dz) {
          // the block's 16 x 16 dz go through the warp's staging rows (stmatrix) and leave
          // as one 16-byte store per lane (a full 32-byte row segment per lane pair)
          const int lr = lm_row(lane);
          const uint32_t ost_w = smem_addr(ost + warp * 512);
          __syncwarp();  // the previous block's staging rows have been read
          stsm_x4(ost_w + lr * 32 + ((((lane >> 4) ^ (lr >> 2)) & 1) << 4), pack_bf16(acc[0][0], acc[0][1]),
                  pack_bf16(acc[0][2], acc[0][3]), pack_bf16(acc[1][0], acc[1][1]), pack_bf16(acc[1][2], acc[1][3]));
          __syncwarp();
          const int row = lane >> 1, half = lane & 1;
          const uint4 v = *reinterpret_cast<const uint4*>(ost + warp * 512 + row * 32 + ((half ^ (row >> 2)) & 1) * 16);
          if (tok0 + 16 * b + row < a.N && col_base + cw + half * 8 < a.Dz)
            *reinterpret_cast<uint4*>(a.dz + (tok0 + 16 * b + row) * a.Dz + col_base + cw + half * 8) = v;
        } else {
          bf16* dz_row = a.dz + (tok0 + 16 * b + g) * a.Dz + col_base + cw + 2 * q;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (tok0 + 16 * b + g + 8 * h < a.N) {
#pragma unroll
              for (int nt = 0; nt < 2; ++nt)
                if (col_base + cw + nt * 8 < a.Dz)
                  *reinterpret_cast<uint32_t*>(dz_row + 8 * h * a.Dz + nt * 8) =
                      pack_bf16(acc[nt][2 * h], acc[nt][2 * h + 1]);
            }
          }
        }
      }
      if (want_dw) {
        // dW^T[col, k] += sum_tok z[tok, col] dl[tok, k]
        uint32_t zt[4];
        const int r = 16 * b + zt_row;
        ldsm_x4_t(z_s + zt_box + r * 128 + (((zt_chunk ^ r) & 7) << 4), zt);
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
          uint32_t db[4];
          ldsm_x4_t(smem_addr(dl_cur + (16 * b + lm_row(lane)) * L::DLB + (kt * 16 + lm_col(lane)) * 2), db);
          mma_bf16(dwa[2 * kt], zt, db[0], db[1]);
          mma_bf16(dwa[2 * kt + 1], zt, db[2], db[3]);
        }
      }
      if (dz_tma) {
        __syncwarp();  // the warp's dW reads of these z rows are done
        const int r = 16 * b + lm_row(lane);
        stsm_x4(z_s + zt_box + r * 128 + (((2 * (warp & 3) + (lane >> 4)) ^ r) & 7) * 16, dzp[0], dzp[1], dzp[2],
                dzp[3]);
      }
    }
    if (dz_tma) {
      fence_proxy_async();  // this thread's dz rows, before the store
      __syncthreads();
      if (threadIdx.x == 0) {
        tma_store_2d(&dzmap, static_cast<int>(col_base), static_cast<int>(tok0), z_s);
        if (col_base + 64 < a.Dz) tma_store_2d(&dzmap, static_cast<int>(col_base) + 64, static_cast<int>(tok0), z_s + L::zbox);
        bulk_commit();
      }
    }
  }
  if (threadIdx.x == 0) bulk_wait<0>();  // the last dz stores
  griddep_launch_dependents();  // only the dW partial store is left
  if (want_dw) {
    const int64_t grp = blockIdx.y;
#pragma unroll
    for (int kn = 0; kn < 2 * KT; ++kn)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = kn * 8 + 2 * q + (e & 1);
        const int64_t col = col_base + cw + g + 8 * (e >> 1);
        if (k < a.K && col < a.Dz) a.dw_part[(grp * a.K + k) * a.Dz + col] = dwa[kn][e];
      }
  }
}

// out[i] = sum over the groups' dW partials (fixed order), four lanes per element
// (quad_part_sum): the sum is short (K x Dz elements) and spread over many partials
__global__ void k_sum_groups(const float* __restrict__ part, int64_t groups, int64_t n, void* out, int dtype) {
  griddep_wait();  // the partials of the backward kernel
  const int sub = threadIdx.x & 3;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x / 4;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 4; i < n; i += step) {
    const float s = quad_part_sum(part, groups, n, i, sub);
    if (sub == 0) st_any(out, dtype, i, s);
  }
  griddep_launch_dependents();
}

int sm_count_r() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Grid of the backward: slices x token groups, one wave of the CTAs an SM holds (four at one
// base group, three at two: the kernel's launch bounds).
void bwd_plan(int64_t N, int64_t Dz, int K, int64_t& slices, int64_t& groups, int64_t& tpg) {
  slices = ceil_div(Dz, kZC);
  const int64_t tiles = std::max<int64_t>(1, ceil_div(N, kBwdTile));
  const int64_t target = static_cast<int64_t>(sm_count_r()) * (K <= 16 ? 4 : 3);
  groups = std::min<int64_t>(tiles, std::max<int64_t>(1, target / slices));
  tpg = ceil_div(tiles, groups);
  groups = ceil_div(tiles, tpg);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int set_smem(const void* kern, bool (&configured)[64], int smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return note_cuda(e);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    // the whole unified L1 / shared array as shared memory, so that as many CTAs as the
    // registers allow are resident (these kernels stage through shared memory, not L1)
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return note_cuda(e);
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  return MOC_OK;
}

template <int KT>
int fwd_kt(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, void* alpha, cudaStream_t st) {
  static bool configured[64] = {};
  int rc = set_smem(reinterpret_cast<const void*>(k_router_fwd_tc<KT>), configured, FwdLayout<KT>::total);
  if (rc != MOC_OK) return rc;
  CUtensorMap zmap, wmap;
  rc = make_tmap_bf16_2d(&zmap, z, static_cast<uint64_t>(Dz), static_cast<uint64_t>(N),
                         static_cast<uint64_t>(Dz) * 2, 64, kFwdRows);
  if (rc != MOC_OK) return rc;
  rc = make_tmap_bf16_2d(&wmap, w, static_cast<uint64_t>(Dz), static_cast<uint64_t>(K), static_cast<uint64_t>(Dz) * 2,
                         64, KT * 16);
  if (rc != MOC_OK) return rc;
  const cudaError_t e = launch_pdl(k_router_fwd_tc<KT>, dim3(static_cast<unsigned>(ceil_div(N, kFwdRows))), dim3(128),
                                   FwdLayout<KT>::total, st, zmap, wmap, static_cast<bf16*>(alpha), N, Dz, K, act);
  note_launch();
  return note_cuda(e);
}

template <int KT>
int bwd_kt(RouterBwdArgs& a, const void* z, int64_t slices, int64_t groups, void* dw, cudaStream_t st) {
  static bool configured[64] = {};
  int rc = set_smem(reinterpret_cast<const void*>(k_router_bwd_tc<KT>), configured, BwdLayout<KT>::total);
  if (rc != MOC_OK) return rc;
  CUtensorMap zmap;
  rc = make_tmap_bf16_2d(&zmap, z, static_cast<uint64_t>(a.Dz), static_cast<uint64_t>(a.N),
                         static_cast<uint64_t>(a.Dz) * 2, 64, kBwdTile);
  if (rc != MOC_OK) return rc;
  // dz: stored from the z area of the stage, kBwdTile rows at a time (a map of z, unused, when
  // there is no dz or it is not 16-byte aligned)
  CUtensorMap dzmap;
  rc = make_tmap_bf16_2d(&dzmap, a.dz != nullptr && a.vec_dz ? static_cast<const void*>(a.dz) : z, static_cast<uint64_t>(a.Dz),
                         static_cast<uint64_t>(a.N), static_cast<uint64_t>(a.Dz) * 2, 64, kBwdTile);
  if (rc != MOC_OK) return rc;
  cudaError_t e = launch_pdl(k_router_bwd_tc<KT>, dim3(static_cast<unsigned>(slices), static_cast<unsigned>(groups)),
                             dim3(256), BwdLayout<KT>::total, st, zmap, dzmap, a);
  note_launch();
  if (e != cudaSuccess) return note_cuda(e);
  if (dw != nullptr) {
    const int64_t n = static_cast<int64_t>(a.K) * a.Dz;
    const int64_t blocks = std::min<int64_t>(ceil_div(4 * n, 256), 8 * sm_count_r());
    e = launch_pdl(k_sum_groups, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, a.dw_part, groups, n, dw,
                   static_cast<int>(MOC_DTYPE_BF16));
    note_launch();
  }
  return note_cuda(e);
}

}  // namespace

bool tc_router_supported(int64_t N, int64_t Dz, int K, int dtype) {
  return dtype == MOC_DTYPE_BF16 && K % 8 == 0 && K <= 32 && Dz % 8 == 0 && N > 0 && ceil_div(Dz, kZC) <= 65535;
}

int tc_router_forward(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, void* alpha,
                      cudaStream_t st) {
  if (!aligned16(z) || !aligned16(w) || (reinterpret_cast<uintptr_t>(alpha) & 3u)) return MOC_ERR_MISALIGNED;
  return K <= 16 ? fwd_kt<1>(N, Dz, K, act, z, w, alpha, st) : fwd_kt<2>(N, Dz, K, act, z, w, alpha, st);
}

size_t tc_router_backward_ws(int64_t N, int64_t Dz, int K) {
  int64_t slices, groups, tpg;
  bwd_plan(N, Dz, K, slices, groups, tpg);
  return align_up(static_cast<size_t>(groups * K * Dz) * sizeof(float), 256);
}

int tc_router_backward(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, const void* alpha,
                       const void* dalpha, int da_dtype, void* dz, void* dw, void* ws, size_t ws_bytes,
                       cudaStream_t st) {
  if (!aligned16(z) || !aligned16(w) || (dz && (reinterpret_cast<uintptr_t>(dz) & 3u))) return MOC_ERR_MISALIGNED;
  if (ws_bytes < tc_router_backward_ws(N, Dz, K)) return MOC_ERR_WORKSPACE_TOO_SMALL;
  if (dz == nullptr && dw == nullptr) return MOC_OK;
  RouterBwdArgs a{};
  a.w = static_cast<const bf16*>(w);
  a.alpha = static_cast<const bf16*>(alpha);
  a.dalpha = dalpha;
  a.da_dtype = da_dtype;
  a.dz = static_cast<bf16*>(dz);
  a.dw_part = dw != nullptr ? static_cast<float*>(ws) : nullptr;
  a.N = N;
  a.Dz = Dz;
  a.K = K;
  a.act = act;
  a.vec_ad = da_dtype == MOC_DTYPE_BF16 && aligned16(alpha) && aligned16(dalpha) && K % 8 == 0;
  a.vec_dz = dz != nullptr && aligned16(dz);
  int64_t slices, groups, tpg;
  bwd_plan(N, Dz, K, slices, groups, tpg);
  a.tiles_per_group = tpg;
  return K <= 16 ? bwd_kt<1>(a, z, slices, groups, dw, st) : bwd_kt<2>(a, z, slices, groups, dw, st);
}

// ------------------------------------------------------------------ no-allocation variant

// Fixed scratch for tc_router_backward_noalloc: the dweight partials of one call.  It is
// part of the library image, so no call allocates; every call reuses (and overwrites) it.
static __device__ __align__(256) float g_noalloc_scratch[MOC_NOALLOC_SCRATCH_BYTES / sizeof(float)];

int tc_router_backward_noalloc(int64_t N, int64_t Dz, int K, int act, const void* z, const void* w, const void* alpha,
                               const void* dalpha, int da_dtype, void* dz, void* dw, cudaStream_t st) {
  if (tc_router_backward_ws(N, Dz, K) > MOC_NOALLOC_SCRATCH_BYTES) return MOC_ERR_SCRATCH_LIMIT;
  // Device address of the array, looked up once per device with that device current
  // (host code cannot use the symbol itself: on the host it names a stand-in, not device memory).
  static std::mutex lock;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return note_cuda(e);
  if (dev < 0 || dev >= 64) return MOC_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> guard(lock);
    if (addr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return note_cuda(e);
      addr[dev] = p;
    }
    scratch = addr[dev];
  }
  // Every dweight partial is written before the reduction reads it, so nothing is cleared.
  return tc_router_backward(N, Dz, K, act, z, w, alpha, dalpha, da_dtype, dz, dw, scratch,
                            MOC_NOALLOC_SCRATCH_BYTES, st);
}

int router_status(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_router_status, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_router_status, &zero, sizeof(int));
    if (e != cudaSuccess) return note_cuda(e);
  }
  *out = v;
  return MOC_OK;
}

int wait_timeout_probe(uint32_t limit, cudaStream_t st) {
  k_wait_timeout_probe<<<1, 1, 0, st>>>(limit);
  note_launch();
  return note_cuda(cudaGetLastError());
}

}  // namespace moc
