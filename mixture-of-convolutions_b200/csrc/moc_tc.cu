// Tensor-core MoC convolution for bf16 x / alpha / basis (sm_100a).
//
// The three K-contractions of the operator are small GEMMs per tile:
//   W[t, s, ch]   = sum_k alpha[t, k] basis[k, s, ch]             (forward, dx, SiLU pre)
//   dalpha[t, k]  = sum_{s,ch} m[t, s, ch] basis[k, s, ch]        (m = dz * x shifted)
//   dbasis[k,s,ch]= sum_t alpha[t, k] m[t, s, ch]
// They run on the tensor cores (mma.sync bf16 -> fp32); the shifts, SiLU and the dz*x
// products run on the CUDA cores in registers, so the per-token kernel W and the product
// m never touch memory.  Rounding points follow the reference's bf16 mode
// (moc/kernels.py:92-95, 125-130, 390-408): alpha, basis and m enter the dots as bf16.
//
// Work decomposition: a CTA owns a 128-channel slice and a contiguous range of 64-token
// work items (fixed-length tiles or the varlen chunks of chunk_indices); 8 warps each own
// 16 channels.  Tiles are staged by TMA (two 64-channel 128B-swizzled boxes of x and dy,
// one dense box of alpha per stage, double buffered on mbarriers, issued by one thread);
// rows that belong to a neighbouring sequence are zeroed in shared memory after landing.
//   forward : y = [silu](sum_s W_s * x_shift_s)                       one pass
//   backward: dz (SiLU pre recomputed on chip), dx, per-slice dalpha partials and per-CTA
//             dbasis partials in one pass over x, dy, alpha; a second small kernel adds the
//             partials in a fixed order (deterministic, no atomics).
// y and dx leave through the stage they were computed from (each 16-row block overwrites
// rows no later block reads) by TMA stores, one per 64-channel box and tile.  Between blocks
// the backward keeps its dbasis accumulators in tensor memory (tcgen05.ld / st per tap).
#include <algorithm>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_mma.cuh"
#include "moc_tma.cuh"

namespace moc {

__device__ int g_conv_status;  // kStatus* bits of bounded waits that ran out

namespace {

constexpr int kTile = 64;              // token rows per work item
constexpr int kBD = 128;               // channels per CTA (two 64-channel TMA boxes)
constexpr int kThreads = 256;          // 8 warps x 16 channels
constexpr int kRowB = (kBD + 8) * 2;   // basis row in smem: 272 B (16 B pad: conflict-free ldmatrix)
constexpr int kHalo = 8;               // past-halo rows kept before each tile (S - 1 <= 7)
constexpr int kFut = 16;               // future rows kept after each tile (S - 1 <= 7, one 16-row block)

constexpr int align1k(int v) { return (v + 1023) / 1024 * 1024; }

// ---- TMEM as the home of the backward's dbasis accumulators.  Each warp owns 8 S KT fp32
// columns of its 32-lane quarter; a tap's 8 KT values per lane are loaded, advanced by
// mma.sync and stored back once per 16-token block, so they take registers only while used.

__device__ __forceinline__ void tm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// one warp: allocate ncols columns (address written to shared memory at slot)
__device__ __forceinline__ void tm_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tm_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// 8 consecutive fp32 columns of this thread's lane <-> v[0..1][0..3]
__device__ __forceinline__ void tm_ld8(uint32_t taddr, float (&v)[2][4]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i >> 2][i & 3] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tm_st8(uint32_t taddr, const float (&v)[2][4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr),
               "r"(__float_as_uint(v[0][0])), "r"(__float_as_uint(v[0][1])), "r"(__float_as_uint(v[0][2])),
               "r"(__float_as_uint(v[0][3])), "r"(__float_as_uint(v[1][0])), "r"(__float_as_uint(v[1][1])),
               "r"(__float_as_uint(v[1][2])), "r"(__float_as_uint(v[1][3]))
               : "memory");
}
// a tap's 2 KT n-tiles of accumulators (8 KT columns); element copies, so v stays in registers
template <int KT>
__device__ __forceinline__ void tm_ld_tap(uint32_t taddr, float (&v)[2 * KT][4]) {
#pragma unroll
  for (int h = 0; h < KT; ++h) {
    float t[2][4];
    tm_ld8(taddr + 8 * h, t);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[2 * h + (i >> 2)][i & 3] = t[i >> 2][i & 3];
  }
}
template <int KT>
__device__ __forceinline__ void tm_st_tap(uint32_t taddr, const float (&v)[2 * KT][4]) {
#pragma unroll
  for (int h = 0; h < KT; ++h) {
    float t[2][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) t[i >> 2][i & 3] = v[2 * h + (i >> 2)][i & 3];
    tm_st8(taddr + 8 * h, t);
  }
}
constexpr int pow2_at_least(int v, int p = 32) { return p >= v ? p : pow2_at_least(v, 2 * p); }

// PART (backward only) selects the work of one launch: kBwdAll (dx, dalpha and dbasis in
// one pass), or, where the dbasis accumulators (S x KP x 16 channels per warp) would leave
// no registers for anything else, two passes: kBwdDxDa (dx, dalpha) and kBwdDb (dbasis).
constexpr int kBwdAll = 0, kBwdDxDa = 1, kBwdDb = 2;
constexpr bool bwd_split(int KT, int S) { return KT * S > 8; }

template <int KT, int S, bool ACT, bool BWD, int PART = kBwdAll>
struct Layout {
  static constexpr int KP = KT * 16;  // bases padded to the MMA K
  // basis fragments live in registers where they fit beside the accumulators (<= 4 (tap,
  // 16-base) groups), and in the dx / dalpha pass of a split backward (no dbasis
  // accumulators, one CTA per SM by shared memory either way), where reading them from
  // shared memory every tap would bound the pass
  static constexpr bool BREG = KT * S <= 4 || PART == kBwdDxDa;
  static constexpr int XR = kHalo + kTile + ((BWD && ACT) ? kFut : 0);  // x rows per stage
  // rows of dy / alpha after the tile start: the dx taps read up to S-1 <= 7 future rows;
  // with SiLU the pre-activation of those rows is one more 16-row MMA block.
  static constexpr int FR = BWD ? (ACT ? kTile + kFut : kTile + 8) : 0;
  static constexpr int AR = BWD ? (ACT ? kTile + kFut : kTile + 8) : kTile;
  static constexpr int ARB = KP * 2;  // dense alpha rows
  static constexpr int xbox = XR * 128;
  static constexpr int dybox = FR * 128;
  static constexpr int x_bytes = 2 * xbox;
  static constexpr int dy_bytes = 2 * dybox;
  static constexpr int a_bytes = align1k(AR * ARB);
  static constexpr int stage_bytes = x_bytes + dy_bytes + a_bytes;
  static constexpr int tx_bytes = x_bytes + dy_bytes + AR * ARB;
  static constexpr int basis_bytes = S * KP * kRowB;
  // dalpha partials of RB 16-row blocks x 8 warps, reduced across warps once per RB blocks
  // (with the basis staged beside them at 32 bases and more than 4 taps: one block)
  // (SiLU backward at one base group: two, so that two CTAs fit an SM)
  static constexpr int RB = (KT == 1 || BREG) ? ((BWD && ACT) ? 2 : 4) : (S > 4 ? 1 : 2);
  static constexpr int red_bytes = (BWD && PART != kBwdDb) ? RB * 8 * 16 * KP * 4 : 0;
  // with register-resident basis fragments the basis staging area is reused for the
  // dalpha reduction buffer once the fragments are loaded
  // the forward stages its basis through the stage buffers, a few taps per pass, before the
  // first tile is loaded, and keeps its fragments in registers afterwards: at 32 bases and more
  // than 4 taps (up to 68 KB) so that two CTAs fit an SM, at one base group and up to 4 taps
  // so that four fit (45 KB and 64 registers each)
  static constexpr bool BALIAS = !BWD && (KT * S > 8 || (KT == 1 && S <= 4));
  static constexpr int head_bytes =
      BALIAS ? 0
             : align1k((BWD && BREG) ? (basis_bytes > red_bytes ? basis_bytes : red_bytes) : basis_bytes + red_bytes);
  // per-warp output staging: one 16-row x 16-channel bf16 block (32-byte rows)
  static constexpr int ost_bytes = BWD ? 0 : 8 * 16 * 32;
  // (the SiLU backward needs no staging of its own: it writes dz, bf16, over dy in the tile)
  // SiLU backward: the dz rows an item hands to the item before it (up to 7 rows x 128 channels)
  static constexpr int carry_bytes = (BWD && ACT) ? 8 * kBD * 2 : 0;
  static constexpr int total = 1024 + 2 * stage_bytes + head_bytes + carry_bytes + ost_bytes + 64;
  static constexpr int min_blocks = BWD ? ((BREG && KT == 1) ? 2 : 1) : ((KT == 1 && S <= 4) ? 4 : 2);
};

struct TcArgs {
  RowMap rm;
  int64_t D;
  int K;
  const bf16* basis;
  bf16* out;
  bf16* dx;
  float* da_part;  // [n_slices][n_tokens][K]
  float* db_part;  // [groups][K][S][D]
  int64_t items_per_group;
  int64_t n_tokens;
};

// lane -> row / column offsets of the four 8x8 matrices of an ldmatrix.x4 covering a
// 16(rows) x 16(cols) block: matrix i = lane/8 holds rows (i&1)*8.. and cols (i>>1)*8..
__device__ __forceinline__ int lm_row(int lane) { return (lane & 7) + ((lane >> 3) & 1) * 8; }
__device__ __forceinline__ int lm_col(int lane) { return (lane >> 4) * 8; }

// Byte offset of 16-byte chunk `chunk` of alpha row `row` in a stage: the TMA box has rows of
// ARB = 32 or 64 bytes written with the swizzle of that span, so that the 8 rows an ldmatrix
// matrix reads fall on distinct banks (dense 32-byte rows would pair them two-way).  The
// swizzle repeats every 8 rows, so row 16 b + r is 16 b ARB bytes past row r: callers add
// that part separately and keep this one free of the block index.
template <class L>
__device__ __forceinline__ uint32_t alpha_off(int row, int chunk) {
  const int sw = L::ARB == 32 ? (row >> 2) & 1 : (row >> 1) & 3;
  return static_cast<uint32_t>(row * L::ARB + ((chunk ^ sw) << 4));
}

// Float offset of column `col` of row `row` (of 16) in a warp's dalpha reduction rows: the
// 8-float groups are permuted per row so that a warp's float2 stores to its 8 rows spread
// over all banks (rows of 16 or 32 floats would otherwise map rows onto the same banks).
template <int KP>
__device__ __forceinline__ int red_off(int row, int col) {
  const int f = KP == 16 ? ((row >> 1) & 1) : (row & 3);
  return row * KP + (col ^ (f << 3));
}

// Shared-memory carve-up, common to both kernels.
template <class L>
struct Smem {
  uint32_t stages;  // 2 stages, 1024-byte aligned
  char* stages_p;
  char* head;       // basis staging / dalpha reduction
  char* carry;      // SiLU backward: dz rows handed from one item to the next
  char* ost;        // per-warp output staging
  uint32_t bar;     // 2 mbarriers
  __device__ explicit Smem(char* raw) {
    char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    stages_p = base;
    stages = smem_addr(base);
    head = base + 2 * L::stage_bytes;
    carry = head + L::head_bytes;
    ost = carry + L::carry_bytes;
    bar = smem_addr(ost + L::ost_bytes);
  }
};

// taps [s0, s0 + ns) of the basis slice into rows (s - s0) * KP + k of basis_s
template <class L, bool BWD>
__device__ __forceinline__ void load_basis(const TcArgs& a, char* basis_s, int64_t ch_base, int S, int s0 = 0,
                                           int ns = -1) {
  constexpr int KP = L::KP;
  if (ns < 0) ns = S;
  for (int idx = threadIdx.x; idx < ns * KP * 16; idx += kThreads) {
    const int row = idx >> 4, chunk = idx & 15;
    const int s = s0 + row / KP, k = row - (s - s0) * KP;
    const int64_t ch = ch_base + chunk * 8;
    const bool ok = k < a.K && ch < a.D;
    const bf16* src = ok ? a.basis + (static_cast<int64_t>(k) * S + s) * a.D + ch : a.basis;
    cp_async16(smem_addr(basis_s + row * kRowB + chunk * 16), src, ok ? 16u : 0u);
  }
}

// Thread 0: stage `stage` <- tile starting at token r0 (x from r0 - kHalo), channel slice ch_base.
template <class L, bool BWD>
__device__ __forceinline__ void issue_tile(const CUtensorMap* xm, const CUtensorMap* dym, const CUtensorMap* am,
                                           uint32_t stage, uint32_t bar, int64_t r0, int64_t ch_base) {
  fence_proxy_async();
  mbar_expect_tx(bar, L::tx_bytes);
  const int c0 = static_cast<int>(ch_base);
  const int row = static_cast<int>(r0);
  tma_load_2d(stage, xm, c0, row - kHalo, bar);
  tma_load_2d(stage + L::xbox, xm, c0 + 64, row - kHalo, bar);
  if constexpr (BWD) {
    tma_load_2d(stage + L::x_bytes, dym, c0, row, bar);
    tma_load_2d(stage + L::x_bytes + L::dybox, dym, c0 + 64, row, bar);
  }
  tma_load_2d(stage + L::x_bytes + L::dy_bytes, am, 0, row, bar);
}

// Zeroes rows [0, zx) of the x tile and rows [zdy, FR) of the dy tile (whole 128-byte
// rows of both boxes): taps and gradients must not see a neighbouring sequence.
template <class L>
__device__ __forceinline__ void zero_rows(char* stage, int zx, int zdy) {
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int idx = threadIdx.x; idx < zx * 16; idx += kThreads) {
    const int row = idx >> 4, part = idx & 15;
    *reinterpret_cast<uint4*>(stage + (part >> 3) * L::xbox + row * 128 + (part & 7) * 16) = z;
  }
  const int ndy = L::FR - zdy;
  for (int idx = threadIdx.x; idx < ndy * 16; idx += kThreads) {
    const int row = zdy + (idx >> 4), part = idx & 15;
    *reinterpret_cast<uint4*>(stage + L::x_bytes + (part >> 3) * L::dybox + row * 128 + (part & 7) * 16) = z;
  }
}

// Fills the x-tile rows of the tokens ss-1 .. ss-(S-1) before the sequence from the
// attached cache (prefill with a cache); called after zero_rows, between CTA barriers.
template <class L>
__device__ __forceinline__ void fill_halo(char* stage, const RowMap& rm, int64_t ss, int64_t r0, int64_t ch_base,
                                          int64_t D, int S) {
  for (int idx = threadIdx.x; idx < (S - 1) * kBD; idx += kThreads) {
    const int m = idx / kBD + 1, ch = idx - (m - 1) * kBD;
    const int64_t row = ss - m - (r0 - kHalo);
    const int64_t gch = ch_base + ch;
    if (row < 0 || row >= L::XR || gch >= D) continue;
    const int r = static_cast<int>(row), c64 = ch & 63;
    *reinterpret_cast<bf16*>(stage + (ch >> 6) * L::xbox + r * 128 + ((((c64 >> 3) ^ r) & 7) << 4) + (c64 & 7) * 2) =
        __float2bfloat16_rn(rm.halo_at(ss, ss - m, gch));
  }
}

// ------------------------------------------------------------------ forward

template <int KT, int S, bool ACT>
__global__ void __launch_bounds__(kThreads, (Layout<KT, S, ACT, false>::min_blocks))
    k_tc_fwd(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap amap,
             const __grid_constant__ CUtensorMap ymap, TcArgs a) {
  using L = Layout<KT, S, ACT, false>;
  extern __shared__ __align__(1024) char smem_raw[];
  const Smem<L> sm(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ch_base = static_cast<int64_t>(blockIdx.x) * kBD;
  const int64_t n_items = a.rm.n_items();
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * a.items_per_group;
  const int64_t i1 = i0 + a.items_per_group < n_items ? i0 + a.items_per_group : n_items;
  if (i0 >= i1) return;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&xmap);
    tma_prefetch_desc(&amap);
    mbar_init(sm.bar, 1);
    mbar_init(sm.bar + 8, 1);
    fence_mbar_init();
  }
  uint32_t bw[S][KT][4];  // basis fragments for W = alpha . basis_s (B operand, 2 channel n-tiles)
  if constexpr (L::BALIAS) {
    constexpr int TPP = (2 * L::stage_bytes) / (L::KP * kRowB);  // taps per pass through the stages
#pragma unroll
    for (int s0 = 0; s0 < S; s0 += TPP) {
      load_basis<L, false>(a, sm.stages_p, ch_base, S, s0, s0 + TPP < S ? TPP : S - s0);
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
#pragma unroll
      for (int ds = 0; ds < TPP; ++ds)
#pragma unroll
        for (int kt = 0; kt < KT; ++kt)
          if (s0 + ds < S)
            ldsm_x4_t(smem_addr(sm.stages_p + (ds * L::KP + kt * 16 + lm_row(lane)) * kRowB +
                                (warp * 16 + lm_col(lane)) * 2),
                      bw[s0 + ds < S ? s0 + ds : 0][kt]);
      __syncthreads();  // the stages are reused for the next pass / the tiles
    }
  } else {
    load_basis<L, false>(a, sm.head, ch_base, S);
    cp_async_commit();
  }
  griddep_wait();  // x and alpha may come from the kernels before this one
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t ss, se, r0, r1;
    if (a.rm.item(i0, ss, se, r0, r1))
      issue_tile<L, false>(&xmap, nullptr, &amap, sm.stages, sm.bar, r0, ch_base);
    else
      mbar_arrive(sm.bar);
  }

  // per-lane constants of the swizzled ldmatrix addresses: this warp's 16 channels are
  // 16-byte chunks 2*(warp&3) + {0,1} of box warp>>2
  const uint32_t x_box = static_cast<uint32_t>((warp >> 2) * L::xbox);
  const int x_chunk = 2 * (warp & 3) + (lane >> 4);
  const int lrow = lm_row(lane);
  const int64_t ch_stage = ch_base + warp * 16;  // the warp's first channel
  const uint32_t ost_w = smem_addr(sm.ost + warp * 512);

  for (int64_t it = i0; it < i1; ++it) {
    const int cur = static_cast<int>((it - i0) & 1);
    const uint32_t parity = static_cast<uint32_t>(((it - i0) >> 1) & 1);
    const bool landed = mbar_wait(sm.bar + 8 * cur, parity);
    if (__syncthreads_or(!landed)) {
      if (threadIdx.x == 0) {
        atomicOr(&g_conv_status, kStatusWaitTimeout);
        mbar_wait(sm.bar + 8 * cur, parity);
        bulk_wait<0>();
      }
      return;
    }
    // every thread is past tile it-1, so its stage can be refilled with tile it+1 once the
    // y store of tile it-1 has read it
    if (threadIdx.x == 0 && it + 1 < i1) {
      int64_t ss, se, r0, r1;
      const uint32_t nbar = sm.bar + 8 * (cur ^ 1);
      bulk_wait_read<0>();
      if (a.rm.item(it + 1, ss, se, r0, r1))
        issue_tile<L, false>(&xmap, nullptr, &amap, sm.stages + (cur ^ 1) * L::stage_bytes, nbar, r0, ch_base);
      else
        mbar_arrive(nbar);
    }
    if constexpr (!L::BALIAS) {
      if (it == i0) {
        cp_async_wait<0>();
        __syncthreads();
#pragma unroll
        for (int s = 0; s < S; ++s)
#pragma unroll
          for (int kt = 0; kt < KT; ++kt)
            ldsm_x4_t(smem_addr(sm.head + (s * L::KP + kt * 16 + lrow) * kRowB + (warp * 16 + lm_col(lane)) * 2),
                      bw[s][kt]);
      }
    }
    if (it + 1 == i1) griddep_launch_dependents();  // the CTA's last item
    int64_t ss, se, r0, r1;
    if (a.rm.item(it, ss, se, r0, r1)) {
      char* stage_p = sm.stages_p + cur * L::stage_bytes;
      const int zx = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ss - (r0 - kHalo), 0), L::XR));
      if (zx > 0) {  // uniform across the CTA
        zero_rows<L>(stage_p, zx, L::FR);
        __syncthreads();
        if (a.rm.halo != nullptr) {
          fill_halo<L>(stage_p, a.rm, ss, r0, ch_base, a.D, S);
          __syncthreads();
        }
      }
      const uint32_t x_s = sm.stages + cur * L::stage_bytes;
      const uint32_t a_s = x_s + L::x_bytes;
      const int rows = static_cast<int>(r1 - r0);
      const int nb = (rows + 15) >> 4;
      // y of a whole tile leaves through the stage: block b's outputs overwrite x rows 16 b ..
      // 16 b + 15 of this warp's columns, which only blocks up to b read (block b + 1 starts
      // at row 16 b + 17), and one TMA store per box writes the tile.  Shorter items store
      // through the warp's staging rows.
      const bool y_tma = rows == kTile;  // uniform across the CTA
      bf16* out_tile = a.out + r0 * a.D + ch_stage;
#pragma unroll 1
      for (int b = 0; b < nb; ++b) {
        uint32_t af[KT][4];
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) ldsm_x4(a_s + (16 * b) * L::ARB + alpha_off<L>(lrow, 2 * kt + (lane >> 4)), af[kt]);
        float acc[2][4] = {};
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const int j = S - 1 - s;
          float w[2][4];
          mma_bf16_z(w[0], af[0], bw[s][0][0], bw[s][0][1]);
          mma_bf16_z(w[1], af[0], bw[s][0][2], bw[s][0][3]);
#pragma unroll
          for (int kt = 1; kt < KT; ++kt) {
            mma_bf16(w[0], af[kt], bw[s][kt][0], bw[s][kt][1]);
            mma_bf16(w[1], af[kt], bw[s][kt][2], bw[s][kt][3]);
          }
          uint32_t xr[4];
          // row kHalo + 16 b - j + lrow: a 16-row step is 2048 bytes and leaves the swizzle term alone
          const int xrow0 = kHalo - j + lrow;
          ldsm_x4(x_s + x_box + xrow0 * 128 + (((x_chunk ^ xrow0) & 7) << 4) + b * 2048, xr);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            ffma2(acc[nt][0], acc[nt][1], w[nt][0], w[nt][1], bf_lo(xr[2 * nt]), bf_hi(xr[2 * nt]));
            ffma2(acc[nt][2], acc[nt][3], w[nt][2], w[nt][3], bf_lo(xr[2 * nt + 1]), bf_hi(xr[2 * nt + 1]));
          }
        }
        // the block's 16 x 16 outputs go through the warp's staging rows (stmatrix) and
        // leave as one full 32-byte row segment per lane pair
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int nt = i >> 1, h = i & 1;
          float v0 = acc[nt][2 * h], v1 = acc[nt][2 * h + 1];
          if (ACT) {
            const float2 sv = silu_bf2(v0, v1);
            v0 = sv.x;
            v1 = sv.y;
          }
          o[i] = pack_bf16(v0, v1);
        }
        __syncwarp();  // the previous block's staging rows / this block's x rows have been read
        if (y_tma) {
          const int yr = 16 * b + lrow;
          stsm_x4(x_s + x_box + yr * 128 + (((x_chunk ^ yr) & 7) << 4), o[0], o[1], o[2], o[3]);
          continue;
        }
        stsm_x4(ost_w + lrow * 32 + ((((lane >> 4) ^ (lrow >> 2)) & 1) << 4), o[0], o[1], o[2], o[3]);
        __syncwarp();
        {
          const int row = lane >> 1, half = lane & 1;
          const uint4 v = *reinterpret_cast<const uint4*>(sm.ost + warp * 512 + row * 32 + ((half ^ (row >> 2)) & 1) * 16);
          if (16 * b + row < rows && ch_stage + half * 8 < a.D)
            *reinterpret_cast<uint4*>(out_tile + (16 * b + row) * a.D + half * 8) = v;
        }
      }
      if (y_tma) {
        fence_proxy_async();  // this thread's y rows, before the store
        __syncthreads();
        if (threadIdx.x == 0) {
          tma_store_2d(&ymap, static_cast<int>(ch_base), static_cast<int>(r0), x_s);
          if (ch_base + 64 < a.D) tma_store_2d(&ymap, static_cast<int>(ch_base) + 64, static_cast<int>(r0), x_s + L::xbox);
          bulk_commit();
        }
      }
    }
  }
  if (threadIdx.x == 0) bulk_wait<0>();  // the last y stores
}

// ------------------------------------------------------------------ backward

template <int KT, int S, bool ACT, int PART>
__global__ void __launch_bounds__(kThreads, (Layout<KT, S, ACT, true, PART>::min_blocks))
    k_tc_bwd(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap dymap,
             const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap dxmap, TcArgs a) {
  using L = Layout<KT, S, ACT, true, PART>;
  constexpr int KP = L::KP;
  constexpr bool BREG = L::BREG;
  constexpr bool DXDA = PART != kBwdDb;  // this launch computes dx and dalpha
  constexpr bool DB = PART != kBwdDxDa;  // this launch computes dbasis
  // dbasis accumulators live in TMEM (8 S KT columns per warp, two warps per lane quarter)
  constexpr int kTmWarpCols = 8 * S * KT;
  constexpr int kTmCols = pow2_at_least(2 * kTmWarpCols);
  // one base group and at most 4 taps: the per-tap ldmatrix offsets are kept per lane and the
  // four 16-token blocks of an item are unrolled (the registers the TMEM accumulators free)
  constexpr bool kLean = KT == 1 && S <= 4;
  extern __shared__ __align__(1024) char smem_raw[];
  const Smem<L> sm(smem_raw);
  char* basis_s = sm.head;
  float* red_s = reinterpret_cast<float*>(sm.head + (BREG ? 0 : L::basis_bytes));  // [RB][8 warps][16][KP]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t slice = blockIdx.x;
  const int64_t ch_base = slice * kBD;
  const int64_t n_items = a.rm.n_items();
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * a.items_per_group;
  const int64_t i1 = i0 + a.items_per_group < n_items ? i0 + a.items_per_group : n_items;
  const bool want_dx = DXDA && a.dx != nullptr;
  const int ch_w = warp * 16;  // this warp's channel offset inside the slice
  // With SiLU the CTA runs its items last to first.  The dx taps of an item read dz up to S - 1
  // rows past its end, which are the first rows of the next item: computed there already (its
  // pre-activation, from the same x, alpha and basis, in the same order), they are handed over
  // through `sm.carry` instead of being recomputed as a fifth 16-row block.
  auto item_of = [&](int64_t it) { return ACT ? i0 + i1 - 1 - it : it; };
  int64_t prev_ss = -1, prev_r0 = -1;  // sequence start and first row of the item run before

  // per-lane constants: basis rows (padded, unswizzled), alpha rows (dense), and the
  // swizzled x / dy boxes holding this warp's 16 channels (chunks 2*(warp&3)+{0,1})
  const uint32_t basis_base = smem_addr(basis_s);
  const int lrow = lm_row(lane);
  const uint32_t bt_lane = static_cast<uint32_t>(lrow * kRowB + (ch_w + lm_col(lane)) * 2);
  const uint32_t bn_lane =
      static_cast<uint32_t>(((lane & 7) + (lane >> 4) * 8) * kRowB + (ch_w + ((lane >> 3) & 1) * 8) * 2);
  const uint32_t x_box = static_cast<uint32_t>((warp >> 2) * L::xbox);
  const uint32_t dy_box = static_cast<uint32_t>(L::x_bytes + (warp >> 2) * L::dybox);
  const int m_chunk = 2 * (warp & 3) + (lane >> 4);
  // per-tap lane offsets (a 16-row block step adds 2048 bytes and leaves the swizzle term alone):
  // dz rows t + j, x rows kHalo + t - j, alpha rows t + j (dx) and t (the SiLU pre-activation)
  uint32_t dyo[kLean ? S : 1], xo[kLean ? S : 1], ao[kLean ? S : 1], a0o = 0;
  if constexpr (kLean) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int j = S - 1 - s, rd = j + lrow, rx = kHalo - j + lrow;
      dyo[s] = dy_box + static_cast<uint32_t>(rd * 128 + (((m_chunk ^ rd) & 7) << 4));
      xo[s] = x_box + static_cast<uint32_t>(rx * 128 + (((m_chunk ^ rx) & 7) << 4));
      ao[s] = alpha_off<L>(j + lrow, lane >> 4);
    }
    a0o = alpha_off<L>(lrow, lane >> 4);
  }
  uint32_t tcol = 0;  // this warp's first TMEM accumulator column
  // shared-memory word that receives the TMEM address (beside the mbarriers)
  auto tm_slot = [&]() { return reinterpret_cast<uint32_t*>(sm.ost + L::ost_bytes + 16); };

  uint32_t bw[BREG ? S : 1][KT][4];  // basis, B operand of W = alpha . basis_s
  uint32_t bd[BREG ? S : 1][KT][4];  // basis^T, B operand of dalpha = m . basis_s^T

  if (i0 < i1) {
    if (threadIdx.x == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&dymap);
      tma_prefetch_desc(&amap);
      mbar_init(sm.bar, 1);
      mbar_init(sm.bar + 8, 1);
      fence_mbar_init();
    }
    load_basis<L, true>(a, basis_s, ch_base, S);
    cp_async_commit();
    if constexpr (DB) {
      if (warp == 0) {
        tm_alloc(smem_addr(tm_slot()), kTmCols);
        tm_fence_before();
      }
    }
    griddep_wait();  // x, dy and alpha may come from the kernels before this one
    __syncthreads();
    if constexpr (DB) {
      tm_fence_after();
      tcol = *reinterpret_cast<volatile uint32_t*>(tm_slot()) + (static_cast<uint32_t>(32 * (warp & 3)) << 16) +
             static_cast<uint32_t>((warp >> 2) * kTmWarpCols);
      const float zero[2 * KT][4] = {};
#pragma unroll
      for (int s = 0; s < S; ++s) tm_st_tap<KT>(tcol + 8 * KT * s, zero);
    }
    if (threadIdx.x == 0) {
      int64_t ss, se, r0, r1;
      if (a.rm.item(item_of(i0), ss, se, r0, r1))
        issue_tile<L, true>(&xmap, &dymap, &amap, sm.stages, sm.bar, r0, ch_base);
      else
        mbar_arrive(sm.bar);
    }
  } else {
    griddep_wait();  // a CTA without items still writes its (zero) dbasis partial
  }
  for (int64_t it = i0; it < i1; ++it) {
    const int cur = static_cast<int>((it - i0) & 1);
    const uint32_t parity = static_cast<uint32_t>(((it - i0) >> 1) & 1);
    const bool landed = mbar_wait(sm.bar + 8 * cur, parity);
    if (__syncthreads_or(!landed)) {
      if (threadIdx.x == 0) {
        atomicOr(&g_conv_status, kStatusWaitTimeout);
        mbar_wait(sm.bar + 8 * cur, parity);
        bulk_wait<0>();
      }
      if constexpr (DB) {  // the accumulators are given back before the CTA leaves
        tm_wait_st();
        tm_fence_before();
        __syncthreads();
        if (warp == 0) {
          tm_fence_after();
          tm_dealloc(*reinterpret_cast<volatile uint32_t*>(tm_slot()), kTmCols);
        }
      }
      return;
    }
    // every thread is past tile it-1, so its stage can be refilled with tile it+1 once the
    // dx store of tile it-1 has read it
    if (threadIdx.x == 0 && it + 1 < i1) {
      int64_t ss, se, r0, r1;
      const uint32_t nbar = sm.bar + 8 * (cur ^ 1);
      if constexpr (DXDA) bulk_wait_read<0>();
      if (a.rm.item(item_of(it + 1), ss, se, r0, r1))
        issue_tile<L, true>(&xmap, &dymap, &amap, sm.stages + (cur ^ 1) * L::stage_bytes, nbar, r0, ch_base);
      else
        mbar_arrive(nbar);
    }
    if (it == i0) {
      cp_async_wait<0>();
      __syncthreads();
      if constexpr (BREG) {
#pragma unroll
        for (int s = 0; s < (BREG ? S : 1); ++s)
#pragma unroll
          for (int kt = 0; kt < KT; ++kt) {
            ldsm_x4_t(basis_base + (s * KP + kt * 16) * kRowB + bt_lane, bw[s][kt]);
            ldsm_x4(basis_base + (s * KP + kt * 16) * kRowB + bn_lane, bd[s][kt]);
          }
        __syncthreads();  // the basis area becomes the dalpha reduction buffer
      }
    }
    int64_t ss, se, r0, r1;
    const bool valid = a.rm.item(item_of(it), ss, se, r0, r1);
    char* stage_p = sm.stages_p + cur * L::stage_bytes;
    const uint32_t x_s = sm.stages + cur * L::stage_bytes;
    const uint32_t a_s = x_s + L::x_bytes + L::dy_bytes;
    const int rows = valid ? static_cast<int>(r1 - r0) : 0;
    // dx of a whole tile leaves through the stage: block b's dx overwrites its dy rows (this
    // warp's columns, which no later block reads), and one TMA store per box writes the tile.
    // Shorter items store from registers.
    const bool dx_tma = want_dx && rows == kTile;  // uniform across the CTA
    if (valid) {
      const int zx = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ss - (r0 - kHalo), 0), L::XR));
      const int zdy = static_cast<int>(std::min<int64_t>(std::max<int64_t>(se - r0, 0), L::FR));
      if (zx > 0 || zdy < L::FR) {  // uniform across the CTA
        zero_rows<L>(stage_p, zx, zdy);
        __syncthreads();
        if (zx > 0 && a.rm.halo != nullptr) {
          fill_halo<L>(stage_p, a.rm, ss, r0, ch_base, a.D, S);
          __syncthreads();
        }
      }
    }

    // swizzled shared address of the ldmatrix row of this lane at tile row `row0 + lrow`
    auto x_addr = [&](int row0) {
      const int r = row0 + lrow;
      return x_s + x_box + r * 128 + (((m_chunk ^ r) & 7) << 4);
    };
    auto dy_addr = [&](int row0) {
      const int r = row0 + lrow;
      return x_s + dy_box + r * 128 + (((m_chunk ^ r) & 7) << 4);
    };
    // alpha fragments (the A operand of W) of tile rows ar .. ar + 15
    auto alpha_frag = [&](int ar, uint32_t (&af)[KT][4], uint32_t lean_off) {
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        if constexpr (kLean)  // KT == 1: lean_off is the lane's offset of rows (ar & 15) + lrow
          ldsm_x4(a_s + (ar & ~15) * L::ARB + lean_off, af[kt]);
        else
          ldsm_x4(a_s + (ar & ~15) * L::ARB + alpha_off<L>((ar & 15) + lrow, 2 * kt + (lane >> 4)), af[kt]);
      }
    };
    // W fragments (C layout) of tap s from alpha fragments
    auto w_of = [&](const uint32_t (&afs)[KT][4], int s, float (&w)[2][4]) {
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        const uint32_t(&af)[4] = afs[kt];
        uint32_t b0, b1, b2, b3;
        if constexpr (BREG) {
          b0 = bw[s][kt][0], b1 = bw[s][kt][1], b2 = bw[s][kt][2], b3 = bw[s][kt][3];
        } else {
          uint32_t bf[4];
          ldsm_x4_t(basis_base + (s * KP + kt * 16) * kRowB + bt_lane, bf);
          b0 = bf[0], b1 = bf[1], b2 = bf[2], b3 = bf[3];
        }
        if (kt == 0) {
          mma_bf16_z(w[0], af, b0, b1);
          mma_bf16_z(w[1], af, b2, b3);
        } else {
          mma_bf16(w[0], af, b0, b1);
          mma_bf16(w[1], af, b2, b3);
        }
      }
    };
    // W fragments for alpha rows starting at tile row ar, tap s
    auto w_frag = [&](int ar, int s, float (&w)[2][4], uint32_t lean_off) {
      uint32_t af[KT][4];
      alpha_frag(ar, af, lean_off);
      w_of(af, s, w);
    };

    if (valid) {
      // ---- phase 1 (SiLU): dz = dy * silu'(pre) for tile rows 0..79 (future rows feed dx),
      // rounded to bf16 and written over dy in the stage (each lane its own pairs), so phase 2
      // is the plain backward on dz
      if constexpr (ACT) {
        // the next item (run just before this one) continues this item's sequence: its first
        // S - 1 dz rows are this item's rows kTile.., kept in sm.carry
        const bool carried = prev_ss == ss && prev_r0 == r1 && r1 < se && r1 - r0 == kTile;  // uniform
        const int nb1 = carried ? 4 : 5;
        for (int b = 0; b < nb1; ++b) {
          float pre[2][4] = {};
          if (16 * b < se - r0) {
            uint32_t af[KT][4];  // the block's own alpha rows serve every tap
            alpha_frag(16 * b, af, a0o);
#pragma unroll
            for (int s = 0; s < S; ++s) {
              const int j = S - 1 - s;
              float w[2][4];
              w_of(af, s, w);
              uint32_t xr[4];
              if constexpr (kLean)
                ldsm_x4(x_s + xo[s] + b * 2048, xr);
              else
                ldsm_x4(x_addr(kHalo + 16 * b - j), xr);
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                ffma2(pre[nt][0], pre[nt][1], w[nt][0], w[nt][1], bf_lo(xr[2 * nt]), bf_hi(xr[2 * nt]));
                ffma2(pre[nt][2], pre[nt][3], w[nt][2], w[nt][3], bf_lo(xr[2 * nt + 1]), bf_hi(xr[2 * nt + 1]));
              }
            }
          }
          // dy of the block in the fragment order of pre (register 2 nt + h: rows g + 8 h,
          // channels 8 nt + 2 q, + 1), times silu'(pre), back over dy
          uint32_t d[4];
          ldsm_x4(dy_addr(16 * b), d);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float2 ds = dsilu_bf2(pre[nt][2 * h], pre[nt][2 * h + 1]);
              const float2 o = __fmul2_rn(make_float2(bf_lo(d[2 * nt + h]), bf_hi(d[2 * nt + h])), ds);
              d[2 * nt + h] = pack_bf16(o.x, o.y);
            }
          stsm_x4(dy_addr(16 * b), d[0], d[1], d[2], d[3]);
        }
        __syncwarp();
        // the warp's 16 channels of rows 0 .. S - 2 (two 16-byte chunks a row): lane 2 r + hf
        // takes the carried rows into rows kTile + r, then leaves its own rows r for the item
        // that runs next (the same words of sm.carry, read before they are written)
        if (lane < 2 * (S - 1)) {
          const int r = lane >> 1, chunk = 2 * (warp & 3) + (lane & 1);
          uint4* cw = reinterpret_cast<uint4*>(sm.carry + r * (kBD * 2) + (ch_w + 8 * (lane & 1)) * 2);
          if (carried) {
            const int row = kTile + r;
            *reinterpret_cast<uint4*>(stage_p + dy_box + row * 128 + (((chunk ^ row) & 7) << 4)) = *cw;
          }
          *cw = *reinterpret_cast<const uint4*>(stage_p + dy_box + r * 128 + (((chunk ^ r) & 7) << 4));
        }
        __syncwarp();
      }
    }

    // ---- phase 2: per 16-row block: dx, m = dz * x_shift, dalpha, dbasis
    const int nb = (rows + 15) >> 4;  // uniform across the CTA
    // one 16-token block of the item (b < nb)
    auto block = [&](const int b) {
      uint32_t ab[DB ? KT : 1][4];  // alpha as the B operand of dbasis (tokens x bases)
      if constexpr (DB) {
#pragma unroll
        for (int kt = 0; kt < KT; ++kt)
          ldsm_x4_t(a_s + (16 * b) * L::ARB + alpha_off<L>(lrow, 2 * kt + (lane >> 4)), ab[kt]);
      }
      uint32_t dyu[4];  // dz (= dy without SiLU) of this block, packed bf16 pairs
      ldsm_x4(dy_addr(16 * b), dyu);
      if constexpr (DB) tm_wait_st();  // the previous block's accumulator stores
      float dxa[2][4] = {};
      float daa[2 * KT][4] = {};
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const int j = S - 1 - s;
        if (want_dx) {
          float w[2][4];
          w_frag(16 * b + j, s, w, kLean ? ao[s] : 0u);  // W at rows t + j
          uint32_t dys[4];
          if constexpr (kLean)
            ldsm_x4(x_s + dyo[s] + b * 2048, dys);
          else
            ldsm_x4(dy_addr(16 * b + j), dys);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            ffma2(dxa[nt][0], dxa[nt][1], w[nt][0], w[nt][1], bf_lo(dys[2 * nt]), bf_hi(dys[2 * nt]));
            ffma2(dxa[nt][2], dxa[nt][3], w[nt][2], w[nt][3], bf_lo(dys[2 * nt + 1]), bf_hi(dys[2 * nt + 1]));
          }
        }
        uint32_t xr[4];
        if constexpr (kLean)
          ldsm_x4(x_s + xo[s] + b * 2048, xr);
        else
          ldsm_x4(x_addr(kHalo + 16 * b - j), xr);
        uint32_t m[4];  // A operand (tokens x channels) of dalpha, rounded to bf16
#pragma unroll
        for (int r = 0; r < 4; ++r) m[r] = hmul2_bf16(dyu[r], xr[r]);
        if constexpr (DXDA) {
#pragma unroll
          for (int kt = 0; kt < KT; ++kt) {
            if constexpr (BREG) {
              mma_bf16(daa[2 * kt], m, bd[s][kt][0], bd[s][kt][1]);
              mma_bf16(daa[2 * kt + 1], m, bd[s][kt][2], bd[s][kt][3]);
            } else {
              uint32_t bb[4];
              ldsm_x4(basis_base + (s * KP + kt * 16) * kRowB + bn_lane, bb);
              mma_bf16(daa[2 * kt], m, bb[0], bb[1]);
              mma_bf16(daa[2 * kt + 1], m, bb[2], bb[3]);
            }
          }
        }
        if constexpr (DB) {
          float acc[2 * KT][4];  // this tap's dbasis^T accumulators, from TMEM
          tm_ld_tap<KT>(tcol + 8 * KT * s, acc);
          uint32_t mt[4] = {movm_t(m[0]), movm_t(m[2]), movm_t(m[1]), movm_t(m[3])};
          tm_wait_ld();
#pragma unroll
          for (int kt = 0; kt < KT; ++kt) {
            mma_bf16(acc[2 * kt], mt, ab[kt][0], ab[kt][1]);
            mma_bf16(acc[2 * kt + 1], mt, ab[kt][2], ab[kt][3]);
          }
          tm_st_tap<KT>(tcol + 8 * KT * s, acc);
        }
      }
      if (dx_tma) {
        __syncwarp();  // the warp's reads of these dy rows are done
        stsm_x4(dy_addr(16 * b), pack_bf16(dxa[0][0], dxa[0][1]), pack_bf16(dxa[0][2], dxa[0][3]),
                pack_bf16(dxa[1][0], dxa[1][1]), pack_bf16(dxa[1][2], dxa[1][3]));
      } else if (want_dx) {
        bf16* dx_row = a.dx + (r0 + 16 * b + g) * a.D + ch_base + ch_w + 2 * q;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (16 * b + g + 8 * h < rows) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
              if (ch_base + ch_w + nt * 8 < a.D)
                *reinterpret_cast<uint32_t*>(dx_row + 8 * h * a.D + nt * 8) =
                    pack_bf16(dxa[nt][2 * h], dxa[nt][2 * h + 1]);
          }
        }
      }
      // dalpha partial of this warp's 16 channels -> red_s[b % RB][warp]; the CTA adds the
      // 8 warps once every RB blocks (and after the tile's last block)
      if constexpr (!DXDA) return;
      float* red = red_s + ((b % L::RB) * 8 + warp) * 16 * KP;
#pragma unroll
      for (int kn = 0; kn < 2 * KT; ++kn)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          *reinterpret_cast<float2*>(red + red_off<KP>(g + 8 * h, kn * 8 + 2 * q)) =
              make_float2(daa[kn][2 * h], daa[kn][2 * h + 1]);
      if (b % L::RB == L::RB - 1 || b == nb - 1) {
        if (dx_tma && b == nb - 1) fence_proxy_async();  // this thread's dx rows, before the store
        __syncthreads();
        if (dx_tma && b == nb - 1 && threadIdx.x == 0) {
          tma_store_2d(&dxmap, static_cast<int>(ch_base), static_cast<int>(r0), x_s + L::x_bytes);
          if (ch_base + 64 < a.D)
            tma_store_2d(&dxmap, static_cast<int>(ch_base) + 64, static_cast<int>(r0), x_s + L::x_bytes + L::dybox);
          bulk_commit();
        }
        // four consecutive bases of one token row per thread: 16-byte loads of the 8 warps'
        // partials (red_off keeps aligned groups of four together), added in warp order
        const int b0 = b - b % L::RB;
        const int n_out = (b - b0 + 1) * 16 * KP;
        for (int o = 4 * threadIdx.x; o < n_out; o += 4 * kThreads) {
          const int blk = o / (16 * KP), rem = o - blk * 16 * KP;
          const int row = rem / KP, k = rem - row * KP;
          const float* rb = red_s + blk * 8 * 16 * KP + red_off<KP>(row, k);
          float4 sum = *reinterpret_cast<const float4*>(rb);
#pragma unroll
          for (int w = 1; w < 8; ++w) {
            const float4 v = *reinterpret_cast<const float4*>(rb + w * 16 * KP);
            const float2 lo = __fadd2_rn(make_float2(sum.x, sum.y), make_float2(v.x, v.y));
            const float2 hi = __fadd2_rn(make_float2(sum.z, sum.w), make_float2(v.z, v.w));
            sum = make_float4(lo.x, lo.y, hi.x, hi.y);
          }
          const int trow = 16 * (b0 + blk) + row;
          // K % 8 == 0 on this path: a group of four is all valid or all padding
          if (k < a.K && trow < rows)
            *reinterpret_cast<float4*>(a.da_part + (slice * a.n_tokens + r0 + trow) * a.K + k) = sum;
        }
        if (b < nb - 1) __syncthreads();  // red_s is rewritten by the next blocks of this tile
      }
    };
    if constexpr (kLean) {  // the four blocks unrolled
#pragma unroll
      for (int b = 0; b < kTile / 16; ++b)
        if (b < nb) block(b);
    } else {
#pragma unroll 1
      for (int b = 0; b < nb; ++b) block(b);
    }
    if constexpr (ACT) {
      prev_ss = valid ? ss : -1;
      prev_r0 = valid ? r0 : -1;
    }
    // the next iteration's wait barrier orders these reads of red_s and the stage before reuse
  }

  if (DXDA && threadIdx.x == 0) bulk_wait<0>();  // the last dx stores
  griddep_launch_dependents();  // only the dbasis partial store is left
  // dbasis partial of this CTA: db_part[group][k][s][ch]
  if constexpr (!DB) return;
  float dba[DB ? S : 1][2 * KT][4] = {};  // dbasis^T: (ch g | g+8) x (k 8kn + 2q..), from TMEM
  if (i0 < i1) {
    tm_wait_st();
#pragma unroll
    for (int s = 0; s < S; ++s) tm_ld_tap<KT>(tcol + 8 * KT * s, dba[s]);
    tm_wait_ld();
    tm_fence_before();
    __syncthreads();
    if (warp == 0) {
      tm_fence_after();
      tm_dealloc(*reinterpret_cast<volatile uint32_t*>(tm_slot()), kTmCols);
    }
  }
  const int64_t grp = blockIdx.y;
#pragma unroll
  for (int s = 0; s < (DB ? S : 1); ++s)
#pragma unroll
    for (int kn = 0; kn < 2 * KT; ++kn)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = kn * 8 + 2 * q + (e & 1);
        const int64_t ch = ch_base + ch_w + g + 8 * (e >> 1);
        if (k < a.K && ch < a.D) a.db_part[((grp * a.K + k) * S + s) * a.D + ch] = dba[s][kn][e];
      }
}

// dalpha[i] = sum over channel slices, dbasis[i] = sum over token groups (fixed order).
__global__ void k_tc_finalize(const float* __restrict__ da_part, int64_t n_slices, int64_t nk, void* dalpha,
                              int adt, const float* __restrict__ db_part, int64_t groups, int64_t ksd, void* dbasis,
                              int bdt) {
  griddep_wait();  // the partials of the backward kernel
  const int64_t total = nk + ksd;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    if (i < nk) {
#pragma unroll 8
      for (int64_t c = 0; c < n_slices; ++c) s += __ldg(da_part + c * nk + i);
      st_any(dalpha, adt, i, s);
    } else {
      const int64_t j = i - nk;
#pragma unroll 8
      for (int64_t g = 0; g < groups; ++g) s += __ldg(db_part + g * ksd + j);
      st_any(dbasis, bdt, j, s);
    }
  }
  griddep_launch_dependents();
}

// ------------------------------------------------------------------ host side

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

struct Plan {
  RowMap rm;
  int64_t slices, groups, ipg;
};

Plan make_plan(const moc_problem& p, int ctas_per_sm) {
  Plan pl;
  pl.rm = make_rowmap(p, kTile);
  pl.slices = ceil_div(p.dim, kBD);
  const int64_t items = pl.rm.n_items();
  const int64_t target = static_cast<int64_t>(sm_count()) * ctas_per_sm;
  int64_t groups = std::max<int64_t>(1, target / pl.slices);
  groups = std::min<int64_t>(groups, std::max<int64_t>(items, 1));
  pl.ipg = std::max<int64_t>(1, ceil_div(items, groups));
  pl.groups = std::max<int64_t>(1, ceil_div(items, pl.ipg));
  return pl;
}

// Raises the dynamic shared-memory limit of `kern` once per device (`configured` is owned
// by the caller's template instantiation, i.e. one flag set per kernel), so launches
// captured into a CUDA graph later make no attribute calls.
int configure(const void* kern, bool (&configured)[64], int smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return note_cuda(e);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return note_cuda(e);
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  return MOC_OK;
}

struct Maps {
  CUtensorMap x, dy, a, out;  // out: the TMA-stored output, dx (backward) or y (forward)
};

template <class L, bool BWD>
int make_maps(const moc_problem& p, const void* x, const void* dy, const void* alpha, const void* dx, Maps& m) {
  const uint64_t D = static_cast<uint64_t>(p.dim), N = static_cast<uint64_t>(p.n_tokens);
  int rc = make_tmap_bf16_2d(&m.x, x, D, N, D * 2, 64, L::XR, 128);
  if (rc == MOC_OK && BWD) rc = make_tmap_bf16_2d(&m.dy, dy, D, N, D * 2, 64, L::FR, 128);
  // dx: stored from the dy area of the stage, 64 rows at a time (a map of dy when there is no dx)
  if (rc == MOC_OK && BWD) rc = make_tmap_bf16_2d(&m.out, dx != nullptr ? dx : dy, D, N, D * 2, 64, kTile, 128);
  if (rc == MOC_OK)  // alpha rows of KP bases (32 or 64 bytes), swizzled over their span
    rc = make_tmap_bf16_2d(&m.a, alpha, static_cast<uint64_t>(p.n_bases), N, static_cast<uint64_t>(p.n_bases) * 2,
                           L::KP, L::AR, L::ARB);
  return rc;
}

template <int KT, int S, bool ACT>
int fwd_inst(const moc_problem& p, TcArgs& args, const void* x, const void* alpha, cudaStream_t st) {
  using L = Layout<KT, S, ACT, false>;
  const Plan pl = make_plan(p, L::min_blocks);
  args.rm = pl.rm;
  args.items_per_group = pl.ipg;
  if (pl.rm.n_items() == 0) return MOC_OK;
  static bool configured[64] = {};
  int rc = configure(reinterpret_cast<const void*>(k_tc_fwd<KT, S, ACT>), configured, L::total);
  if (rc != MOC_OK) return rc;
  Maps m;
  rc = make_maps<L, false>(p, x, nullptr, alpha, nullptr, m);
  // y: stored from the x area of the stage, 64 rows at a time
  if (rc == MOC_OK)
    rc = make_tmap_bf16_2d(&m.out, args.out, static_cast<uint64_t>(p.dim), static_cast<uint64_t>(p.n_tokens),
                           static_cast<uint64_t>(p.dim) * 2, 64, kTile, 128);
  if (rc != MOC_OK) return rc;
  const cudaError_t e = launch_pdl(k_tc_fwd<KT, S, ACT>, dim3(static_cast<unsigned>(pl.slices), static_cast<unsigned>(pl.groups)),
                                   dim3(kThreads), L::total, st, m.x, m.a, m.out, args);
  note_launch();
  return note_cuda(e);
}

template <int KT, int S, bool ACT>
int bwd_inst(const moc_problem& p, TcArgs& args, const void* x, const void* alpha, const void* dy, void* dalpha,
             void* dbasis, cudaStream_t st) {
  // the layout of the launch (of the first pass when split); both passes share one plan
  using L = Layout<KT, S, ACT, true, bwd_split(KT, S) ? kBwdDxDa : kBwdAll>;
  static_assert(L::min_blocks == ((L::BREG && KT == 1) ? 2 : 1), "bwd_min_blocks() mirrors Layout::min_blocks");
  const Plan pl = make_plan(p, L::min_blocks);
  args.rm = pl.rm;
  args.items_per_group = pl.ipg;
  const int64_t nk = p.n_tokens * p.n_bases;
  const int64_t ksd = static_cast<int64_t>(p.n_bases) * p.kernel_size * p.dim;
  // the attribute calls come first: they also make the device's primary context current,
  // which the tensor-map encoding (a driver call) needs
  int rc = MOC_OK;
  if constexpr (bwd_split(KT, S)) {
    using LB = Layout<KT, S, ACT, true, kBwdDb>;
    static_assert(LB::min_blocks == 1, "one plan for both passes");
    static bool conf_a[64] = {}, conf_b[64] = {};
    rc = configure(reinterpret_cast<const void*>(k_tc_bwd<KT, S, ACT, kBwdDxDa>), conf_a, L::total);
    if (rc == MOC_OK) rc = configure(reinterpret_cast<const void*>(k_tc_bwd<KT, S, ACT, kBwdDb>), conf_b, LB::total);
  } else {
    static bool configured[64] = {};
    rc = configure(reinterpret_cast<const void*>(k_tc_bwd<KT, S, ACT, kBwdAll>), configured, L::total);
  }
  if (rc != MOC_OK) return rc;
  Maps m;
  rc = make_maps<L, true>(p, x, dy, alpha, args.dx, m);
  if (rc != MOC_OK) return rc;
  const dim3 grid(static_cast<unsigned>(pl.slices), static_cast<unsigned>(pl.groups));
  if constexpr (bwd_split(KT, S)) {
    rc = note_cuda(launch_pdl(k_tc_bwd<KT, S, ACT, kBwdDxDa>, grid, dim3(kThreads), L::total, st, m.x, m.dy, m.a, m.out, args));
    note_launch();
    if (rc != MOC_OK) return rc;
    rc = note_cuda(launch_pdl(k_tc_bwd<KT, S, ACT, kBwdDb>, grid, dim3(kThreads), Layout<KT, S, ACT, true, kBwdDb>::total,
                              st, m.x, m.dy, m.a, m.out, args));
  } else {
    rc = note_cuda(launch_pdl(k_tc_bwd<KT, S, ACT, kBwdAll>, grid, dim3(kThreads), L::total, st, m.x, m.dy, m.a, m.out, args));
  }
  note_launch();
  if (rc != MOC_OK) return rc;
  return tc_finalize(args.da_part, pl.slices, nk, dalpha, p.alpha_dtype, args.db_part, pl.groups, ksd, dbasis,
                     p.basis_dtype, st);
}

template <template <int, int, bool> class F, typename... Args>
int dispatch(const moc_problem& p, Args&&... args) {
  const int KT = p.n_bases <= 16 ? 1 : 2;
  const bool act = p.activation != 0;
#define MOC_TC_CASE(kt, s)                                           \
  if (KT == kt && p.kernel_size == s)                                \
    return act ? F<kt, s, true>::run(p, std::forward<Args>(args)...) \
               : F<kt, s, false>::run(p, std::forward<Args>(args)...);
  MOC_TC_CASE(1, 1) MOC_TC_CASE(1, 2) MOC_TC_CASE(1, 3) MOC_TC_CASE(1, 4)
  MOC_TC_CASE(1, 5) MOC_TC_CASE(1, 6) MOC_TC_CASE(1, 7) MOC_TC_CASE(1, 8)
  MOC_TC_CASE(2, 1) MOC_TC_CASE(2, 2) MOC_TC_CASE(2, 3) MOC_TC_CASE(2, 4)
  MOC_TC_CASE(2, 5) MOC_TC_CASE(2, 6) MOC_TC_CASE(2, 7) MOC_TC_CASE(2, 8)
#undef MOC_TC_CASE
  return MOC_ERR_UNSUPPORTED_SHAPE;
}

template <int KT, int S, bool ACT>
struct FwdRun {
  static int run(const moc_problem& p, TcArgs& args, const void* x, const void* alpha, cudaStream_t st) {
    return fwd_inst<KT, S, ACT>(p, args, x, alpha, st);
  }
};
template <int KT, int S, bool ACT>
struct BwdRun {
  static int run(const moc_problem& p, TcArgs& args, const void* x, const void* alpha, const void* dy, void* da,
                 void* db, cudaStream_t st) {
    return bwd_inst<KT, S, ACT>(p, args, x, alpha, dy, da, db, st);
  }
};

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Resident backward CTAs per SM for problem p (Layout::min_blocks of the instantiation
// dispatch() selects); the workspace size and the launch must agree on it.
int bwd_min_blocks(const moc_problem& p) {
  const int kt = p.n_bases <= 16 ? 1 : 2;
  const bool breg = kt * p.kernel_size <= 4;
  return (breg && kt == 1) ? 2 : 1;
}

void ws_split(const moc_problem& p, int64_t& slices, int64_t& groups, size_t& da_bytes, size_t& db_bytes) {
  const Plan pl = make_plan(p, bwd_min_blocks(p));
  slices = pl.slices;
  groups = pl.groups;
  da_bytes = align_up(static_cast<size_t>(slices * p.n_tokens * p.n_bases) * sizeof(float), 256);
  db_bytes = align_up(static_cast<size_t>(groups * p.n_bases * p.kernel_size * p.dim) * sizeof(float), 256);
}

}  // namespace

int tc_finalize(const float* da_part, int64_t n_slices, int64_t nk, void* dalpha, int adt, const float* db_part,
                int64_t groups, int64_t ksd, void* dbasis, int bdt, cudaStream_t st) {
  const int64_t blocks = std::min<int64_t>(ceil_div(nk + ksd, 256), 8 * sm_count());
  const cudaError_t e = launch_pdl(k_tc_finalize, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, da_part,
                                   n_slices, nk, dalpha, adt, db_part, groups, ksd, dbasis, bdt);
  note_launch();
  return note_cuda(e);
}

// Whether the shapes tc5_supported() covers take the tcgen05 backward (moc_bwd5.cu); off,
// they take the two-pass warp-level backward below (moc_set_kernel_path(MOC_PATH_WARP_BACKWARD)).
static bool g_bwd5_allowed = true;
void tc_allow_bwd5(bool allowed) { g_bwd5_allowed = allowed; }
static bool use_bwd5(const moc_problem& p) { return g_bwd5_allowed && tc5_supported(p); }

bool tc_conv_supported(const moc_problem& p) {
  if (p.x_dtype != MOC_DTYPE_BF16 || p.alpha_dtype != MOC_DTYPE_BF16 || p.basis_dtype != MOC_DTYPE_BF16) return false;
  if (p.n_bases % 8 != 0 || p.n_bases > 32) return false;
  if (p.kernel_size < 1 || p.kernel_size > 8) return false;
  if (p.dim % 8 != 0) return false;
  if (p.cu_seqlens != nullptr && p.chunk_size != kTile) return false;
  if (ceil_div(p.dim, kBD) > 65535) return false;
  // TMA coordinates are 32-bit
  if (p.n_tokens > (int64_t{1} << 31) - 1024 || p.dim > (int64_t{1} << 31) - 1024) return false;
  return true;
}

int tc_forward(const moc_problem& p, const void* x, const void* alpha, const void* basis, void* out,
               cudaStream_t st) {
  if (!aligned16(x) || !aligned16(alpha) || !aligned16(basis) || !aligned16(out)) return MOC_ERR_MISALIGNED;
  TcArgs args{};
  args.D = p.dim;
  args.K = p.n_bases;
  args.basis = static_cast<const bf16*>(basis);
  args.out = static_cast<bf16*>(out);
  args.n_tokens = p.n_tokens;
  return dispatch<FwdRun>(p, args, x, alpha, st);
}

size_t tc_backward_ws(const moc_problem& p) {
  if (use_bwd5(p)) return tc5_backward_ws(p);
  int64_t slices, groups;
  size_t da, db;
  ws_split(p, slices, groups, da, db);
  return da + db;
}

int tc_backward(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy, void* dx,
                void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!aligned16(ws)) return MOC_ERR_MISALIGNED;  // the dalpha partials are written 16 bytes at a time
  if (use_bwd5(p)) return tc5_backward(p, x, alpha, basis, dy, dx, dalpha, dbasis, ws, ws_bytes, st);
  if (!aligned16(x) || !aligned16(alpha) || !aligned16(basis) || !aligned16(dy) || (dx && !aligned16(dx)))
    return MOC_ERR_MISALIGNED;
  int64_t slices, groups;
  size_t da, db;
  ws_split(p, slices, groups, da, db);
  if (ws_bytes < da + db) return MOC_ERR_WORKSPACE_TOO_SMALL;
  TcArgs args{};
  args.D = p.dim;
  args.K = p.n_bases;
  args.basis = static_cast<const bf16*>(basis);
  args.dx = static_cast<bf16*>(dx);
  args.da_part = static_cast<float*>(ws);
  args.db_part = reinterpret_cast<float*>(static_cast<char*>(ws) + da);
  args.n_tokens = p.n_tokens;
  return dispatch<BwdRun>(p, args, x, alpha, dy, dalpha, dbasis, st);
}

int conv_status(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_conv_status, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_conv_status, &zero, sizeof(int));
    if (e != cudaSuccess) return note_cuda(e);
  }
  *out = v;
  return MOC_OK;
}

}  // namespace moc
