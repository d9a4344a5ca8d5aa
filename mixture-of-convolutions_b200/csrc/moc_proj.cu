// Fused projection + MoC convolution forward, bf16, on the sm_100a tensor cores (tcgen05).
//
//   y = MoC(h . Wp^T)      h [N, Dm], Wp [D, Dm] (nn.Linear layout), y [N, D]
//
// In the reference's attention block (README.md:115-129) each MoC module convolves one slice
// of the qkv projection.  Here the projection runs as a tcgen05 GEMM and the convolution is
// its epilogue, so the projected x never goes to HBM (the unfused path writes x and reads it
// back: 4 bytes per element).  The projection is rounded to bf16 before the convolution, as
// the reference's bf16 qkv tensor is.
//
// Work decomposition: an m-tile is 128 GEMM rows whose first 8 are the causal halo (the
// tokens before its 120 output rows, recomputed rather than exchanged), so a sequence of T
// tokens takes ceil(T / 120) m-tiles and m-tiles never span two sequences.  The two CTAs of
// a cluster (two SMs) share one tcgen05.mma of M = 256 (each CTA's 128 rows) by N = 256
// output channels: each stages its own h rows and half of the Wp rows (32 KB a stage), so a
// staged byte feeds twice the MMA work of a one-SM 128 x 128 tile.  One persistent cluster
// per SM pair takes tile pairs c, c + clusters, ... with the channel tile innermost, so the
// clusters running together share a few h row tiles and all of Wp stays in L2:
//   warp 0     TMA producer (both CTAs): h and Wp k-blocks (64 columns, 128-byte swizzle)
//              into a 4-stage ring, completing on the leader CTA's stage barrier;
//   warp 1     allocates all 512 TMEM columns in both CTAs (two 128 x 256 fp32 accumulators
//              each); in the leader CTA one thread issues tcgen05.mma.cta_group::2 (M=256,
//              N=256, K=16), committing each stage back to both producers and each finished
//              accumulator to both epilogues (multicast commit; no load uses multicast);
//   warps 4-11 epilogue, in two 128-channel passes per tile: tcgen05.ld the accumulator
//              (warp w reads TMEM lanes 32 (w % 4)..),
//              round to bf16 into a swizzled x tile in shared memory (rows before the
//              sequence start zeroed), release the accumulator, then convolve exactly as the
//              standalone forward does (W_s = alpha . basis_s on mma.sync, FFMA2 taps, fused
//              SiLU) and store y through per-warp staging rows with 16-byte stores.  For
//              training the epilogue also copies the tile's rounded x rows to memory (the
//              input of the convolution backward); inference writes y only.
// The two accumulators let the MMAs of tile i+1 run under the epilogue of tile i; the
// leader reuses an accumulator once both CTAs' epilogues have released it.
//
// Every mbarrier wait is bounded.  A wait that runs out records MOC_STATUS_WAIT_TIMEOUT and
// raises a CTA-wide abort flag; every role then leaves its loop, the producers wait (bounded)
// for the copies they issued, the MMA thread for its MMAs, and both CTAs meet at a cluster
// barrier before the TMEM is freed.
// Epilogue decisions to leave are made together (a barrier reduction), so no warp is left
// at a named barrier.
#include <algorithm>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_mma.cuh"
#include "moc_tma.cuh"

namespace moc {

__device__ int g_proj_status;

namespace {

constexpr int kPM = 128;              // GEMM rows per tile
constexpr int kPHalo = 8;             // of which halo rows (S - 1 <= 7)
constexpr int kPOut = kPM - kPHalo;   // output rows per tile
constexpr int kPN = 256;              // output channels per tile (the MMA's N)
constexpr int kPNH = kPN / 2;         // Wp rows staged by each CTA of the pair
constexpr int kPC = 128;              // channels per epilogue pass (two passes per tile)
constexpr int kPK = 64;               // k per stage: 128-byte rows
constexpr int kPStages = 4;
constexpr int kPThreads = 384;        // 12 warps
constexpr int kPEpiWarp0 = 4;         // epilogue warps 4..11
constexpr int kPEpiThreads = 256;
constexpr int kPATile = kPM * kPK * 2;         // 16 KB: h rows of one stage
constexpr int kPStageBytes = kPATile + kPNH * kPK * 2;  // + 16 KB of Wp rows
constexpr int kPXR = kPM + 16;        // staged x rows: the last 16-row block reads up to 8 past the tile
constexpr int kPXBox = kPXR * 128;    // one 64-channel half of the x tile
constexpr int kPRowB = (kPC + 8) * 2; // basis row in shared memory (padded: conflict-free ldmatrix)
constexpr int kPKP = 16;              // bases padded to the MMA K
constexpr int kPARB = kPKP * 2;       // alpha row bytes
constexpr int kPTmemCols = 2 * kPN;   // two accumulators
constexpr uint32_t kPollAbortEvery = 1024;

template <int S>
struct ProjLayout {
  static constexpr int x_off = kPStages * kPStageBytes;
  static constexpr int a_off = x_off + 2 * kPXBox;
  static constexpr int b_off = a_off + kPM * kPARB;
  static constexpr int o_off = b_off + S * kPKP * kPRowB;
  static constexpr int bar_off = o_off + 8 * 512;
  static constexpr int n_bars = 2 * kPStages + 4 + 1;  // full, empty, acc full x2, acc empty x2, drain
  static constexpr int misc_off = bar_off + 8 * n_bars;  // tmem slot, abort flag
  static constexpr int total = 1024 + misc_off + 16;
};

// one module: its rows of the weight, its router output, basis and output
struct ProjMod {
  const bf16* alpha;
  const bf16* basis;
  bf16* y;
  bf16* x;          // optional: the rounded projection, kept for the backward
  int64_t dout;     // channels
  int64_t row_off;  // first weight row
  int64_t tile0;    // first channel tile (over all modules)
  int K, act;
};

struct ProjArgs {
  ProjMod mod[MOC_PROJ_MAX_MODULES];
  int n_mod;
  int64_t seq_len, n_tokens, dm;
  int64_t m_per_seq, m_tiles;
  int64_t n_tiles;     // channel tiles over all modules
  int64_t pair_tiles;  // ceil(m_tiles / 2) x n_tiles
};

// ---- tcgen05 / barrier wrappers

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// executed by the same warp of both CTAs of the pair
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T over the CTA pair (A: each CTA's 128 rows, B: each CTA's
// half of the N rows; D: each CTA's TMEM), both K-major bf16, fp32 accumulate; one thread
// of the leader CTA issues
__device__ __forceinline__ void umma_bf16_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// arrives (once) on the mbarrier at this offset in both CTAs of the pair when every MMA this
// thread issued so far has completed
__device__ __forceinline__ void umma_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n" ::"r"(
          bar),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
// ... on the leader's own mbarrier only
__device__ __forceinline__ void umma_commit_self(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// shared::cluster address of the same offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory that completes on a barrier of either CTA of
// the pair (the leader's: the MMA issuer waits for both CTAs' operands there)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(cluster_bar)
      : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// shared-memory matrix descriptor: K-major tile of 128-byte rows written by TMA with the
// 128-byte swizzle (8-row groups 1024 bytes apart); sm_100 descriptor version 1
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
// instruction descriptor: bf16 A and B (K-major), fp32 D, M = 256 (the pair), N = 256
constexpr uint32_t kProjIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kPN >> 3) << 17) |
                                (static_cast<uint32_t>((2 * kPM) >> 4) << 24);

// named barrier over the epilogue warps; the second form also returns whether any of them
// passed `p`
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kPEpiThreads) : "memory"); }
__device__ __forceinline__ bool epi_any(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred q, o;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred o, 1, %2, q;\n selp.u32 %0, 1, 0, o;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(p)), "n"(kPEpiThreads)
      : "memory");
  return r != 0;
}

// bounded wait that also gives up once another role raised the abort flag
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  for (uint32_t i = 0; i < kSpinLimit; i += kPollAbortEvery) {
    if (mbar_wait(bar, parity, kPollAbortEvery)) return true;
    if (*abort_flag) return false;
  }
  return false;
}
__device__ __forceinline__ void raise_abort(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(&g_proj_status, kStatusWaitTimeout);
}

struct TileCoord {
  int64_t n0, m0, row0;  // first output channel (of its module), first output token, first GEMM row (m0 - halo)
  int64_t wrow0;         // first weight row
  int mod;               // module
  int rows;              // output rows of this tile
  bool seq_first;        // the halo rows precede the sequence start
};

// tile pair tp, CTA `rank` of the pair: m-tile 2 (tp / n_tiles) + rank, channel tile
// tp % n_tiles (of the module whose tiles it falls in).  A CTA past the last m-tile stages
// zero rows (coordinates past the end) and stores nothing.
__device__ __forceinline__ TileCoord tile_coord(const ProjArgs& a, int64_t tp, uint32_t rank) {
  TileCoord c;
  const int64_t pm = tp / a.n_tiles, n = tp - pm * a.n_tiles;
  const int64_t m = 2 * pm + rank;
  int mi = 0;
  while (mi + 1 < a.n_mod && n >= a.mod[mi + 1].tile0) ++mi;
  c.mod = mi;
  c.n0 = (n - a.mod[mi].tile0) * kPN;
  c.wrow0 = a.mod[mi].row_off + c.n0;
  if (m >= a.m_tiles) {
    c.m0 = c.row0 = a.n_tokens;
    c.rows = 0;
    c.seq_first = false;
    return c;
  }
  const int64_t seq = m / a.m_per_seq, ci = m - seq * a.m_per_seq;
  c.m0 = seq * a.seq_len + ci * kPOut;
  c.row0 = c.m0 - kPHalo;
  c.rows = static_cast<int>(std::min<int64_t>(kPOut, a.seq_len - ci * kPOut));
  c.seq_first = ci == 0;
  return c;
}

template <int S>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    k_proj_conv(const __grid_constant__ CUtensorMap hmap, const __grid_constant__ CUtensorMap wmap, ProjArgs a) {
  using L = ProjLayout<S>;
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(base);
  char* x_s = base + L::x_off;
  char* a_s = base + L::a_off;
  char* b_s = base + L::b_off;
  char* o_s = base + L::o_off;
  const uint32_t bar_full = sbase + L::bar_off;
  const uint32_t bar_empty = bar_full + 8 * kPStages;
  const uint32_t bar_accf = bar_empty + 8 * kPStages;
  const uint32_t bar_acce = bar_accf + 16;
  const uint32_t bar_drain = bar_acce + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + L::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int64_t total_tiles = a.pair_tiles;
  const int64_t t_begin = blockIdx.x >> 1, t_step = gridDim.x >> 1;
  const int nk = static_cast<int>((a.dm + kPK - 1) / kPK);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&hmap);
    tma_prefetch_desc(&wmap);
    // the accumulator-empty pair is released by both CTAs' epilogues (the leader's is used)
    for (int i = 0; i < L::n_bars; ++i) {
      const uint32_t bar = bar_full + 8 * i;
      mbar_init(bar, bar == bar_acce || bar == bar_acce + 8 ? 2 : 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), kPTmemCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int64_t issued = 0;
      bool ok = true;
      const uint32_t leader_full = peer_addr(bar_full, 0);
      for (int64_t t = t_begin; t < total_tiles && ok; t += t_step) {
        const TileCoord c = tile_coord(a, t, rank);
        for (int kb = 0; kb < nk; ++kb, ++issued) {
          const int s = static_cast<int>(issued % kPStages);
          const uint32_t use = static_cast<uint32_t>(issued / kPStages);
          if (use > 0 && !wait_or_abort(bar_empty + 8 * s, (use & 1) ^ 1, abort_flag)) {
            raise_abort(abort_flag);
            ok = false;
            break;
          }
          const uint32_t dst = sbase + s * kPStageBytes;
          if (rank == 0) mbar_expect_tx(bar_full + 8 * s, 2 * kPStageBytes);  // both CTAs' bytes
          tma_load_2d_pair(dst, &hmap, kb * kPK, static_cast<int>(c.row0), leader_full + 8 * s);
          tma_load_2d_pair(dst + kPATile, &wmap, kb * kPK, static_cast<int>(c.wrow0 + rank * kPNH),
                           leader_full + 8 * s);
        }
      }
      if (!ok) {  // the copies still in flight land before the CTA's shared memory is released
        if (rank == 0) {
          for (int64_t i = std::max<int64_t>(0, issued - kPStages); i < issued; ++i)
            mbar_wait(bar_full + 8 * static_cast<int>(i % kPStages), static_cast<uint32_t>(i / kPStages) & 1);
        } else {  // they complete on the leader's barriers: allow them a bounded time
          for (int i = 0; i < 4096; ++i) __nanosleep(1000);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      int64_t consumed = 0;
      bool ok = true;
      int li = 0;
      for (int64_t t = t_begin; t < total_tiles && ok; t += t_step, ++li) {
        const int buf = li & 1;
        const uint32_t ub = static_cast<uint32_t>(li >> 1);
        if (ub > 0 && !wait_or_abort(bar_acce + 8 * buf, (ub & 1) ^ 1, abort_flag)) {
          raise_abort(abort_flag);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * kPN);
        for (int kb = 0; kb < nk; ++kb, ++consumed) {
          const int s = static_cast<int>(consumed % kPStages);
          if (!wait_or_abort(bar_full + 8 * s, static_cast<uint32_t>(consumed / kPStages) & 1, abort_flag)) {
            raise_abort(abort_flag);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(sbase + s * kPStageBytes);
          const uint64_t bd = sw128_desc(sbase + s * kPStageBytes + kPATile);
#pragma unroll
          for (int k = 0; k < kPK / 16; ++k)  // +32 bytes per K=16 step inside the swizzled rows
            umma_bf16_pair(d, ad + 2 * k, bd + 2 * k, kProjIdesc, (kb | k) != 0);
          umma_commit_both(bar_empty + 8 * s);
        }
        if (ok) umma_commit_both(bar_accf + 8 * buf);
      }
      // every MMA issued has completed before the TMEM is released
      umma_commit_self(bar_drain);
      mbar_wait(bar_drain, 0);
    }
    __syncwarp();
  } else if (warp >= kPEpiWarp0) {
    // ---------------------------------------------------------------- epilogue
    const int e = warp - kPEpiWarp0;        // 16-channel group of the convolution
    const int et = threadIdx.x - kPEpiWarp0 * 32;
    const int quarter = warp & 3;  // a warp reads TMEM lanes 32 (warp id % 4) .. + 31
    const int half = e >> 2;       // and accumulator columns 64 half .. + 63
    const int lrow = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int lcol = (lane >> 4) * 8;
    const uint32_t xs = smem_addr(x_s);
    const uint32_t x_box = static_cast<uint32_t>((e >> 2) * kPXBox);
    const int x_chunk = 2 * (e & 3) + (lane >> 4);
    const uint32_t a_lane = static_cast<uint32_t>(lrow * kPARB + (((lane >> 4) ^ ((lrow >> 2) & 1)) << 4));
    const uint32_t ost_w = smem_addr(o_s + e * 512);
    uint32_t bw[S][4];  // basis fragments of this warp's 16 channels
    int li = 0;
    const uint32_t acce_leader = peer_addr(bar_acce, 0);
    for (int64_t t = t_begin; t < total_tiles; t += t_step, ++li) {
      const TileCoord c = tile_coord(a, t, rank);
      const ProjMod& md = a.mod[c.mod];
      const int buf = li & 1;
      const uint32_t ub = static_cast<uint32_t>(li >> 1);
      // the tile's channels in 128-channel halves (the second only where it has channels)
      const int halves = c.n0 + kPC < md.dout ? 2 : 1;
      // alpha rows of the tile's output tokens
      {
        const int r = et >> 1, chunk = et & 1;
        const bool ok = r < c.rows && chunk * 8 < md.K;
        const bf16* src = ok ? md.alpha + (c.m0 + r) * md.K + chunk * 8 : md.alpha;
        // 32-byte rows with the 16-byte halves swapped every 4 rows: conflict-free ldmatrix
        cp_async16(smem_addr(a_s + r * kPARB + ((chunk ^ ((r >> 2) & 1)) << 4)), src, ok ? 16u : 0u);
      }
      bool ok = true;
      for (int hh = 0; hh < halves; ++hh) {
        const int64_t c0 = c.n0 + hh * kPC;  // first channel of this half
        // the basis slice of the half's channels
        for (int idx = et; idx < S * kPKP * 16; idx += kPEpiThreads) {
          const int row = idx >> 4, chunk = idx & 15;
          const int s = row / kPKP, k = row - s * kPKP;
          const int64_t ch = c0 + chunk * 8;
          const bool in = k < md.K && ch < md.dout;
          const bf16* src = in ? md.basis + (static_cast<int64_t>(k) * S + s) * md.dout + ch : md.basis;
          cp_async16(smem_addr(b_s + row * kPRowB + chunk * 16), src, in ? 16u : 0u);
        }
        cp_async_commit();
        if (hh == 0) {  // the accumulator of this tile
          const bool landed = wait_or_abort(bar_accf + 8 * buf, ub & 1, abort_flag);
          if (epi_any(!landed)) {
            if (et == 0) raise_abort(abort_flag);
            cp_async_wait<0>();
            ok = false;
            break;
          }
          tc_fence_after();
        }
        {
          // TMEM lane 32 quarter + lane = GEMM row r; 64 columns of it -> bf16 x row r
          const int r = 32 * quarter + lane;
          const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quarter) << 16) +
                                 static_cast<uint32_t>(buf * kPN + hh * kPC + 64 * half);
          uint32_t v0[32], v1[32];
          tmem_ld32(taddr, v0);
          tmem_ld32(taddr + 32, v1);
          tmem_ld_wait();
          const bool zero = c.seq_first && r < kPHalo;  // tokens of the previous sequence
          char* row_p = x_s + half * kPXBox + r * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* v = j < 4 ? v0 + 8 * j : v1 + 8 * (j - 4);
            uint4 w;
            w.x = zero ? 0u : pack_bf16(__uint_as_float(v[0]), __uint_as_float(v[1]));
            w.y = zero ? 0u : pack_bf16(__uint_as_float(v[2]), __uint_as_float(v[3]));
            w.z = zero ? 0u : pack_bf16(__uint_as_float(v[4]), __uint_as_float(v[5]));
            w.w = zero ? 0u : pack_bf16(__uint_as_float(v[6]), __uint_as_float(v[7]));
            *reinterpret_cast<uint4*>(row_p + ((j ^ (r & 7)) << 4)) = w;
          }
        }
        if (hh == halves - 1) tc_fence_before();
        cp_async_wait<0>();
        epi_sync();  // x tile, alpha and basis in shared memory
        if (hh == halves - 1 && et == 0) mbar_arrive_cluster(acce_leader + 8 * buf);  // this CTA is done with it
#pragma unroll
        for (int s = 0; s < S; ++s)
          ldsm_x4_t(smem_addr(b_s + (s * kPKP + lrow) * kPRowB + (e * 16 + lcol) * 2), bw[s]);
        if (md.x != nullptr) {
          // training: the half's output rows of the rounded projection go to memory too, as
          // the x the convolution backward reads (16-byte chunks, 16 per 128-channel row)
          bf16* xg = md.x + c.m0 * md.dout + c0;
          for (int idx = et; idx < c.rows * 16; idx += kPEpiThreads) {
            const int r = idx >> 4, chunk = idx & 15;
            if (c0 + chunk * 8 < md.dout) {
              const int xr = kPHalo + r;
              const uint4 v = *reinterpret_cast<const uint4*>(x_s + (chunk >> 3) * kPXBox + xr * 128 +
                                                              (((chunk & 7) ^ (xr & 7)) << 4));
              *reinterpret_cast<uint4*>(xg + static_cast<int64_t>(r) * md.dout + chunk * 8) = v;
            }
          }
        }
        // ---- the convolution of the tile's output rows (x row = output row + halo)
        const int64_t ch_w = c0 + e * 16;
        bf16* out_tile = md.y + c.m0 * md.dout + ch_w;
        const bool act = md.act != 0;
        const int nb = (c.rows + 15) >> 4;
        const uint32_t as = smem_addr(a_s);
#pragma unroll 1
        for (int b = 0; b < nb; ++b) {
          uint32_t af[4];
          ldsm_x4(as + (16 * b) * kPARB + a_lane, af);
          float acc[2][4] = {};
#pragma unroll
          for (int s = 0; s < S; ++s) {
            const int j = S - 1 - s;
            float w[2][4];
            mma_bf16_z(w[0], af, bw[s][0], bw[s][1]);
            mma_bf16_z(w[1], af, bw[s][2], bw[s][3]);
            uint32_t xr[4];
            const int xrow = kPHalo + 16 * b - j + lrow;
            ldsm_x4(xs + x_box + xrow * 128 + (((x_chunk ^ xrow) & 7) << 4), xr);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              ffma2(acc[nt][0], acc[nt][1], w[nt][0], w[nt][1], bf_lo(xr[2 * nt]), bf_hi(xr[2 * nt]));
              ffma2(acc[nt][2], acc[nt][3], w[nt][2], w[nt][3], bf_lo(xr[2 * nt + 1]), bf_hi(xr[2 * nt + 1]));
            }
          }
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int nt = i >> 1, h = i & 1;
            float v0 = acc[nt][2 * h], v1 = acc[nt][2 * h + 1];
            if (act) {
              const float2 sv = silu_bf2(v0, v1);
              v0 = sv.x;
              v1 = sv.y;
            }
            o[i] = pack_bf16(v0, v1);
          }
          __syncwarp();
          stsm_x4(ost_w + lrow * 32 + ((((lane >> 4) ^ (lrow >> 2)) & 1) << 4), o[0], o[1], o[2], o[3]);
          __syncwarp();
          const int row = lane >> 1, hc = lane & 1;
          const uint4 v = *reinterpret_cast<const uint4*>(o_s + e * 512 + row * 32 + ((hc ^ (row >> 2)) & 1) * 16);
          if (16 * b + row < c.rows && ch_w + hc * 8 < md.dout)
            *reinterpret_cast<uint4*>(out_tile + (16 * b + row) * md.dout + hc * 8) = v;
        }
        epi_sync();  // the x tile, alpha and basis are rewritten next
      }
      if (!ok) break;
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  cluster_sync();  // the leader's MMAs into this CTA's TMEM and shared memory are done
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kPTmemCols);
}

template <int S>
int proj_inst(ProjArgs& args, const void* h, const void* weight, int64_t weight_rows, cudaStream_t st) {
  using L = ProjLayout<S>;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return note_cuda(e);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(k_proj_conv<S>), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             L::total);
    if (e != cudaSuccess) return note_cuda(e);
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  CUtensorMap hmap, wmap;
  int rc = make_tmap_bf16_2d(&hmap, h, static_cast<uint64_t>(args.dm), static_cast<uint64_t>(args.n_tokens),
                             static_cast<uint64_t>(args.dm) * 2, kPK, kPM, 128);
  if (rc == MOC_OK)
    rc = make_tmap_bf16_2d(&wmap, weight, static_cast<uint64_t>(args.dm), static_cast<uint64_t>(weight_rows),
                           static_cast<uint64_t>(args.dm) * 2, kPK, kPNH, 128);
  if (rc != MOC_OK) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t clusters = std::min<int64_t>(std::max(sms / 2, 1), args.pair_tiles);
  k_proj_conv<S><<<static_cast<unsigned>(2 * clusters), kPThreads, L::total, st>>>(hmap, wmap, args);
  note_launch();
  return note_cuda(cudaGetLastError());
}

}  // namespace

int proj_forward_multi(int n, const moc_proj_module* mods, void* const* x_out, int64_t batch, int64_t seq_len,
                       int64_t in_dim, int S, const void* h, const void* weight, int64_t weight_rows, cudaStream_t st) {
  ProjArgs a{};
  a.n_mod = n;
  a.seq_len = seq_len;
  a.n_tokens = batch * seq_len;
  a.dm = in_dim;
  a.m_per_seq = ceil_div(seq_len, kPOut);
  a.m_tiles = batch * a.m_per_seq;
  int64_t tiles = 0;
  for (int i = 0; i < n; ++i) {
    ProjMod& m = a.mod[i];
    m.alpha = static_cast<const bf16*>(mods[i].alpha);
    m.basis = static_cast<const bf16*>(mods[i].basis);
    m.y = static_cast<bf16*>(mods[i].out);
    m.x = x_out ? static_cast<bf16*>(x_out[i]) : nullptr;
    m.dout = mods[i].dim;
    m.row_off = mods[i].row_offset;
    m.tile0 = tiles;
    m.K = mods[i].n_bases;
    m.act = mods[i].activation;
    tiles += ceil_div(mods[i].dim, kPN);
  }
  a.n_tiles = tiles;
  a.pair_tiles = ceil_div(a.m_tiles, int64_t{2}) * a.n_tiles;
  if (a.n_tokens == 0 || tiles == 0) return MOC_OK;
  switch (S) {
    case 1: return proj_inst<1>(a, h, weight, weight_rows, st);
    case 2: return proj_inst<2>(a, h, weight, weight_rows, st);
    case 3: return proj_inst<3>(a, h, weight, weight_rows, st);
    case 4: return proj_inst<4>(a, h, weight, weight_rows, st);
    case 5: return proj_inst<5>(a, h, weight, weight_rows, st);
    case 6: return proj_inst<6>(a, h, weight, weight_rows, st);
    case 7: return proj_inst<7>(a, h, weight, weight_rows, st);
    case 8: return proj_inst<8>(a, h, weight, weight_rows, st);
    default: return MOC_ERR_UNSUPPORTED_SHAPE;
  }
}

int proj_status(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_proj_status, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_proj_status, &zero, sizeof(int));
    if (e != cudaSuccess) return note_cuda(e);
  }
  *out = v;
  return MOC_OK;
}

}  // namespace moc
