// Convolution backward for bf16 x / alpha / basis with the two contractions of the product
// m = dz * x_shift on the 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
// It serves the shapes whose dbasis accumulators would not fit in registers beside the rest
// of the warp-level backward (32 bases and more than 4 taps); the
// warp-level kernel in moc_tc.cu serves the others.
//
// Per token t, channel c and tap s (j = S - 1 - s tokens back):
//   m_s[t, c]      = dz[t, c] * x[t - j, c]                        (bf16, the reference's rounding
//                                                                   point, moc/kernels.py:390-392)
//   dalpha[t, k]   = sum_{s, c} m_s[t, c] basis[k, s, c]           (moc/kernels.py:390-406)
//   dbasis[k,s,c]  = sum_t alpha[t, k] m_s[t, c]                   (moc/kernels.py:407-417)
//   dx[t, c]       = sum_s W_s[t + j, c] dz[t + j, c],  W_s = alpha . basis_s   (moc/kernels.py:156-268)
//
// A CTA owns a 128-channel slice and a contiguous run of 64-token work items (fixed-length
// tiles or the varlen chunks of chunk_indices), one CTA per SM:
//   warp 16      TMA producer: x (with an 8-row past halo), dy and alpha of the items ahead into
//                a ring of two or three stages (128-byte swizzled boxes; alpha with the swizzle of
//                its 64-byte rows); it also allocates the tensor memory;
//   warps 17-18  one thread each issues the tcgen05.mma of each tap (two issuers: at these
//                small shapes the issuing thread, sharing its scheduler with compute warps,
//                sets the pace more than the tensor pipe does):
//                  warp 17: dalpha (M = 64 tokens, N = bases, K = the slice's 128 channels,
//                  8 MMAs) into one of three 64 x N accumulators (item number mod 3);
//                  warp 18: dbasis^T (M = 128 channels, N = bases, K = the item's 64 tokens,
//                  4 MMAs) into the tap's accumulator, which lives for the whole CTA;
//   warps 0-15   16 channels each (warps w and w + 8 share a channel group and split the
//                item's four 16-token blocks): per tap, W_s = alpha . basis_s on mma.sync (the
//                basis fragments read from shared memory once per tap), dx += W_s * dz_shift in
//                packed fp32 (FFMA2), m_s = dz * x_shift in packed bf16, and m_s stored with
//                stmatrix into a ring slot that the MMA threads read as their A operand (one
//                layout serves as the K-major A of dalpha and the MN-major A of dbasis).
// Warps 0-3 read each item's dalpha accumulator back two items later (tcgen05.ld; a 64-row
// accumulator occupies lanes 0-15 of each 32-lane quarter) and write the per-slice dalpha
// partial; at the end all compute warps read the dbasis accumulators and write the CTA's
// partial.  The kernel of moc_tc.cu that adds the partials in a fixed order finishes the
// job (deterministic, no atomics).
//
// With SiLU, a first phase recomputes the pre-activation of the item's 80 rows on chip and
// writes dz = dy * silu'(pre), rounded to bf16, over dy in the stage.
//
// Every mbarrier wait is bounded: a wait that runs out records MOC_STATUS_WAIT_TIMEOUT and
// the thread carries on (no role leaves early, so every arrival the others wait for still
// happens and the CTA always reaches its exit); the results of such a call are not valid.
#include <algorithm>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_mma.cuh"
#include "moc_tma.cuh"

namespace moc {

__device__ int g_bwd5_status;

namespace {

constexpr int kT5 = 64;                  // token rows per item
constexpr int kBD5 = 128;                // channels per CTA
constexpr int kCompWarps = 16;
constexpr int kCompThreads = kCompWarps * 32;
constexpr int kProdWarp = 16, kMmaWarpDa = 17, kMmaWarpDb = 18;
constexpr int kThreads5 = kCompThreads + 96;
constexpr int kHalo5 = 8;                // past-halo rows before each item (S - 1 <= 7)
constexpr int kFut5 = 16;                // future rows after it (SiLU: one more 16-row block)
constexpr int kSlotBytes = 2 * kT5 * 128;  // m of one tap: 64 tokens x 128 channels, two 64-channel halves
constexpr int kSlotHalf = kT5 * 128;
constexpr int kSmemMax = 227 * 1024;
// an item's dalpha accumulator is read back while the compute warps work on the item kDaLag
// items later, so that the read does not wait for the item's last MMAs; kDaLag + 1 buffers
constexpr int kDaLag = 2;
constexpr int kDaBufs = kDaLag + 1;

constexpr int align1k5(int v) { return (v + 1023) / 1024 * 1024; }
constexpr int tmem_cols_for(int need) {
  return need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
}

template <int KT, int S, bool ACT>
struct Layout5 {
  static constexpr int KP = KT * 16;            // bases padded to the MMA's K / N
  static constexpr int ARB = KP * 2;            // alpha row bytes (32 or 64)
  static constexpr int XR = kHalo5 + kT5 + (ACT ? kFut5 : 0);
  static constexpr int FR = ACT ? kT5 + kFut5 : kT5 + 8;  // dy / alpha rows: the dx taps read 7 ahead
  static constexpr int AR = FR;
  static constexpr int xbox = XR * 128;
  static constexpr int dybox = FR * 128;
  static constexpr int x_bytes = 2 * xbox;
  static constexpr int dy_bytes = 2 * dybox;
  static constexpr int a_bytes = align1k5(AR * ARB);
  static constexpr int stage_bytes = x_bytes + dy_bytes + a_bytes;
  static constexpr int tx_bytes = x_bytes + dy_bytes + AR * ARB;
  // basis[k, s, slice] as S x 2 halves x KP rows of 128 bytes, 128-byte swizzle: the K-major
  // B operand of dalpha, and (ldmatrix.trans) the B fragments of W = alpha . basis_s
  static constexpr int basis_bytes = S * 2 * KP * 128;
  static constexpr int avail = kSmemMax - 1024 - 512 - basis_bytes;  // for stages and ring slots
  // input stages in flight: three where they fit beside at least two ring slots, else two;
  // ring slots: as many of four as fit
  static constexpr int NST = avail >= 3 * stage_bytes + 2 * kSlotBytes ? 3 : 2;
  static constexpr int NSLOT = std::min(4, (avail - NST * stage_bytes) / kSlotBytes);
  static constexpr int basis_off = NST * stage_bytes;
  static constexpr int ring_off = basis_off + basis_bytes;
  static constexpr int bar_off = ring_off + NSLOT * kSlotBytes;
  // stage_full[NST], stage_empty[NST], ring_full[NSLOT], ring_empty[NSLOT], da_full[kDaBufs],
  // da_empty[kDaBufs], db_done
  static constexpr int n_bars = 2 * NST + 2 * NSLOT + 2 * kDaBufs + 1;
  static constexpr int misc_off = bar_off + 8 * n_bars;  // tensor-memory base address
  static constexpr int total = 1024 + misc_off + 16;
  static constexpr int da_col = 0;             // kDaBufs dalpha accumulators of KP columns
  static constexpr int db_col = kDaBufs * KP;  // S dbasis accumulators of KP columns
  static constexpr int tmem_cols = tmem_cols_for(kDaBufs * KP + S * KP);
  static_assert(NSLOT >= 2, "shared memory for at least two ring slots");
  static_assert(total <= kSmemMax, "shared memory budget");
  static_assert(kDaBufs * KP + S * KP <= 512, "tensor memory budget");
};

struct Bwd5Args {
  RowMap rm;
  int64_t D;
  int K;
  const bf16* basis;
  bf16* dx;
  float* da_part;  // [n_slices][n_tokens][K]
  float* db_part;  // [groups][K][S][D]
  int64_t items_per_group;
  int64_t n_tokens;
};

// ---- tcgen05 wrappers (one CTA per MMA)

__device__ __forceinline__ void tc_fence_before5() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after5() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc1(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc1(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, bf16 in, fp32 accumulate; issued by one thread
__device__ __forceinline__ void umma_bf16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// arrives once on the mbarrier when every MMA this thread issued so far has completed
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32x(uint32_t taddr, uint32_t (&v)[32]) {
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
// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16x(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
template <int KP>
__device__ __forceinline__ void tmem_ld_kp(uint32_t taddr, uint32_t (&v)[KP]) {
  if constexpr (KP == 32) {
    tmem_ld32x(taddr, v);
  } else {
    tmem_ld16x(taddr, v);
  }
}
__device__ __forceinline__ void tmem_ld_wait5() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// Shared-memory matrix descriptors (sm_100, version 1; addresses and strides in bytes).
// K-major, 128-byte swizzle: rows of 128 bytes, 8-row groups `sbo` apart; an MMA reads 32
// bytes (16 bf16) of K from the start address, which may sit 32, 64 or 96 bytes into a row.
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t saddr, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
// MN-major: a row is one K index, `span` bytes (32, 64 or 128, the swizzle width) of M or N,
// 8 rows form an atom; `lbo` is the byte stride between atoms along M / N and `sbo` between
// 8-row groups along K.
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo, int span) {
  const uint64_t layout = span == 128 ? 2 : span == 64 ? 4 : 6;
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46) | (layout << 61);
}
// instruction descriptor of kind::f16: bf16 A and B, fp32 D, A / B K-major (0) or MN-major (1)
constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void comp_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kCompThreads) : "memory"); }

// bounded wait; a wait that runs out is recorded and the caller carries on
__device__ __forceinline__ void wait_rec(uint32_t bar, uint32_t parity) {
  if (!mbar_wait(bar, parity)) atomicOr(&g_bwd5_status, kStatusWaitTimeout);
}

__device__ __forceinline__ int lm_row5(int lane) { return (lane & 7) + ((lane >> 3) & 1) * 8; }

// byte offset of 16-byte chunk `chunk` of alpha row `row` (rows of ARB bytes, swizzled over
// their span as TMA writes them; the pattern repeats every 8 rows)
template <int ARB>
__device__ __forceinline__ uint32_t alpha_off5(int row, int chunk) {
  const int sw = ARB == 32 ? (row >> 2) & 1 : (row >> 1) & 3;
  return static_cast<uint32_t>(row * ARB + ((chunk ^ sw) << 4));
}

template <int KT, int S, bool ACT>
__global__ void __launch_bounds__(kThreads5, 1)
    k_bwd5(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap dymap,
           const __grid_constant__ CUtensorMap amap, Bwd5Args a) {
  using L = Layout5<KT, S, ACT>;
  constexpr int KP = L::KP;
  constexpr int ARB = L::ARB;
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_addr(base);
  const uint32_t basis_s = sb + L::basis_off;
  const uint32_t ring = sb + L::ring_off;
  const uint32_t bar_stage_full = sb + L::bar_off;
  const uint32_t bar_stage_empty = bar_stage_full + 8 * L::NST;
  const uint32_t bar_ring_full = bar_stage_empty + 8 * L::NST;
  const uint32_t bar_ring_empty = bar_ring_full + 8 * L::NSLOT;
  const uint32_t bar_da_full = bar_ring_empty + 8 * L::NSLOT;
  const uint32_t bar_da_empty = bar_da_full + 8 * kDaBufs;
  const uint32_t bar_db_done = bar_da_empty + 8 * kDaBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::misc_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t slice = blockIdx.x;
  const int64_t ch_base = slice * kBD5;
  const int64_t n_items = a.rm.n_items();
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * a.items_per_group;
  const int64_t i1 = std::min<int64_t>(i0 + a.items_per_group, n_items);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&xmap);
    tma_prefetch_desc(&dymap);
    tma_prefetch_desc(&amap);
    for (int i = 0; i < L::NST; ++i) {
      mbar_init(bar_stage_full + 8 * i, 1);
      mbar_init(bar_stage_empty + 8 * i, kCompWarps + 1);  // compute warps + the dbasis issuer (alpha)
    }
    for (int i = 0; i < kDaBufs; ++i) {
      mbar_init(bar_da_full + 8 * i, 1);
      mbar_init(bar_da_empty + 8 * i, 4);  // the four draining warps
    }
    for (int i = 0; i < L::NSLOT; ++i) {
      mbar_init(bar_ring_full + 8 * i, kCompWarps);
      mbar_init(bar_ring_empty + 8 * i, 2);  // both MMA issuers
    }
    mbar_init(bar_db_done, 1);
    fence_mbar_init();
  }
  if (warp < kCompWarps) {
    // the basis slice, S x 2 halves x KP rows x 128 bytes, 128-byte swizzle; bases past K and
    // channels past D read as zero
    for (int idx = threadIdx.x; idx < S * KP * 16; idx += kCompThreads) {
      const int chunk = idx & 15, row = idx >> 4;  // row = s * KP + k
      const int s = row / KP, k = row - s * KP;
      const int half = chunk >> 3, c = chunk & 7;
      const int64_t ch = ch_base + chunk * 8;
      const bool ok = k < a.K && ch < a.D;
      const bf16* src = ok ? a.basis + (static_cast<int64_t>(k) * S + s) * a.D + ch : a.basis;
      cp_async16(basis_s + ((s * 2 + half) * KP + k) * 128 + ((c ^ (k & 7)) << 4), src, ok ? 16u : 0u);
    }
    cp_async_commit();
  }
  if (warp == kProdWarp) tmem_alloc1(smem_addr(tmem_slot), L::tmem_cols);
  griddep_wait();  // x, dy and alpha may come from the kernels before this one
  if (warp < kCompWarps) {
    cp_async_wait<0>();
    fence_proxy_async();  // the basis rows, before the MMAs read them
  }
  tc_fence_before5();
  __syncthreads();
  tc_fence_after5();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      for (int64_t it = i0; it < i1; ++it) {
        const int n = static_cast<int>(it - i0), st = n % L::NST;
        if (n >= L::NST) wait_rec(bar_stage_empty + 8 * st, static_cast<uint32_t>(n / L::NST - 1) & 1);
        const uint32_t stage = sb + st * L::stage_bytes;
        const uint32_t bar = bar_stage_full + 8 * st;
        int64_t ss, se, r0, r1;
        if (a.rm.item(it, ss, se, r0, r1)) {
          fence_proxy_async();
          mbar_expect_tx(bar, L::tx_bytes);
          const int c0 = static_cast<int>(ch_base), row = static_cast<int>(r0);
          tma_load_2d(stage, &xmap, c0, row - kHalo5, bar);
          tma_load_2d(stage + L::xbox, &xmap, c0 + 64, row - kHalo5, bar);
          tma_load_2d(stage + L::x_bytes, &dymap, c0, row, bar);
          tma_load_2d(stage + L::x_bytes + L::dybox, &dymap, c0 + 64, row, bar);
          tma_load_2d(stage + L::x_bytes + L::dy_bytes, &amap, 0, row, bar);
        } else {
          mbar_arrive(bar);  // an empty item: nothing to load
        }
      }
    }
  } else if (warp == kMmaWarpDa) {
    // ------------------------------------------------------------------ dalpha MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_da = idesc_bf16(64, KP, 0, 0);  // m (K-major) x basis_s (K-major)
      uint32_t ring_ctr = 0;
      for (int64_t it = i0; it < i1; ++it) {
        const int n = static_cast<int>(it - i0), buf = n % kDaBufs;
        int64_t ss, se, r0, r1;
        const bool valid = a.rm.item(it, ss, se, r0, r1);
        if (n >= kDaBufs) wait_rec(bar_da_empty + 8 * buf, static_cast<uint32_t>(n / kDaBufs - 1) & 1);
        const uint32_t d_da = tmem + L::da_col + buf * KP;
        for (int s = 0; s < S; ++s, ++ring_ctr) {
          const int slot = static_cast<int>(ring_ctr % L::NSLOT);
          wait_rec(bar_ring_full + 8 * slot, (ring_ctr / L::NSLOT) & 1);
          tc_fence_after5();
          if (valid) {
            // dalpha[t, k] += sum_c m_s[t, c] basis_s[k, c]: 8 steps of 16 channels; a step moves
            // the descriptors' start address (16-byte units) within their 128-byte rows
            const uint64_t a0 = desc_k_sw128(ring + slot * kSlotBytes, 1024);
            const uint64_t b0 = desc_k_sw128(basis_s + s * 2 * KP * 128, 1024);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t da = ((kk >> 2) * kSlotHalf + (kk & 3) * 32) >> 4;
              const uint32_t db = ((kk >> 2) * KP * 128 + (kk & 3) * 32) >> 4;
              umma_bf16(d_da, a0 + da, b0 + db, idesc_da, (s | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit(bar_ring_empty + 8 * slot);
        }
        umma_commit(bar_da_full + 8 * buf);
      }
    }
  } else if (warp == kMmaWarpDb) {
    // ------------------------------------------------------------------ dbasis MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_db = idesc_bf16(128, KP, 1, 1);  // m^T (MN-major) x alpha (MN-major)
      uint32_t ring_ctr = 0;
      bool db_started = false;
      for (int64_t it = i0; it < i1; ++it) {
        const int n = static_cast<int>(it - i0), st = n % L::NST;
        int64_t ss, se, r0, r1;
        const bool valid = a.rm.item(it, ss, se, r0, r1);
        wait_rec(bar_stage_full + 8 * st, static_cast<uint32_t>(n / L::NST) & 1);  // alpha of this item
        const uint64_t b0 = desc_mn(sb + st * L::stage_bytes + L::x_bytes + L::dy_bytes, 0, 8 * ARB, ARB);
        for (int s = 0; s < S; ++s, ++ring_ctr) {
          const int slot = static_cast<int>(ring_ctr % L::NSLOT);
          wait_rec(bar_ring_full + 8 * slot, (ring_ctr / L::NSLOT) & 1);
          tc_fence_after5();
          if (valid) {
            // dbasis^T[c, k] += sum_t m_s[t, c] alpha[t, k]: 4 steps of 16 tokens
            const uint64_t a0 = desc_mn(ring + slot * kSlotBytes, kSlotHalf, 1024, 128);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(tmem + L::db_col + s * KP, a0 + ((kk * 16 * 128) >> 4), b0 + ((kk * 16 * ARB) >> 4),
                        idesc_db, (db_started || kk != 0) ? 1u : 0u);
          }
          umma_commit(bar_ring_empty + 8 * slot);
        }
        if (valid) db_started = true;
        umma_commit(bar_stage_empty + 8 * st);  // this item's alpha has been read
      }
      umma_commit(bar_db_done);
    }
  } else {
    // ------------------------------------------------------------------ compute warps
    const int cg = warp & 7, bp = warp >> 3;  // channel group of 16, block parity
    const int ch_w = cg * 16;
    const int lrow = lm_row5(lane);
    const int lcol_chunk = lane >> 4;                 // matrix i = lane / 8: chunk i >> 1
    const int half = cg >> 2;                         // 64-channel half of the slice
    const int m_chunk = 2 * (cg & 3) + lcol_chunk;    // 16-byte chunk of this lane's row in the half
    const uint32_t x_box = static_cast<uint32_t>(half * L::xbox);
    const uint32_t dy_box = static_cast<uint32_t>(L::x_bytes + half * L::dybox);
    const bool want_dx = a.dx != nullptr;
    const int g = lane >> 2, q = lane & 3;
    // the lane's ldmatrix / stmatrix row at block 0 and tap shift 0 (blocks are 16 rows = 2048
    // bytes of x / dy / m apart, and 16 * ARB bytes of alpha; a 16-row step leaves the
    // 128-byte swizzle term alone, so the per-tap offsets below depend on the tap only)
    const uint32_t row_sw = static_cast<uint32_t>(lrow * 128 + (((m_chunk ^ lrow) & 7) << 4));
    uint32_t ring_ctr = 0;
    bool any_valid = false;
    static_assert(kDaLag == 2, "the items awaiting read-back are indexed by n & 1");
    int64_t prev_r0[kDaLag] = {0, 0};  // first row and rows of the items not yet read back, by n & 1
    int prev_rows[kDaLag] = {0, 0};

    // reads back the dalpha accumulator of item number n (warps 0-3) and writes its partial
    auto drain_dalpha = [&](int n, int64_t r0, int rows) {
      const int buf = n % kDaBufs;
      wait_rec(bar_da_full + 8 * buf, static_cast<uint32_t>(n / kDaBufs) & 1);
      tc_fence_after5();
      uint32_t v[KP];
      tmem_ld_kp<KP>(tmem + (static_cast<uint32_t>(32 * warp) << 16) + L::da_col + buf * KP, v);
      tmem_ld_wait5();
      tc_fence_before5();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_da_empty + 8 * buf);
      const int t = 16 * warp + lane;  // a 64-row accumulator: lanes 0-15 of each quarter
      if (lane < 16 && t < rows) {
        float* dst = a.da_part + (slice * a.n_tokens + r0 + t) * a.K;
#pragma unroll
        for (int k4 = 0; k4 < KP; k4 += 4)
          if (k4 < a.K)
            *reinterpret_cast<float4*>(dst + k4) = make_float4(__uint_as_float(v[k4]), __uint_as_float(v[k4 + 1]),
                                                               __uint_as_float(v[k4 + 2]), __uint_as_float(v[k4 + 3]));
      }
    };

    for (int64_t it = i0; it < i1; ++it) {
      const int n = static_cast<int>(it - i0), st = n % L::NST;
      wait_rec(bar_stage_full + 8 * st, static_cast<uint32_t>(n / L::NST) & 1);
      int64_t ss = 0, se = 0, r0 = 0, r1 = 0;
      const bool valid = a.rm.item(it, ss, se, r0, r1);
      const int rows = valid ? static_cast<int>(r1 - r0) : 0;
      any_valid |= valid;
      char* stage_p = base + st * L::stage_bytes;
      const uint32_t x_s = sb + st * L::stage_bytes;
      const uint32_t a_s = x_s + L::x_bytes + L::dy_bytes;
      if (valid) {
        const int zx = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ss - (r0 - kHalo5), 0), L::XR));
        const int zdy = static_cast<int>(std::min<int64_t>(std::max<int64_t>(se - r0, 0), L::FR));
        if (zx > 0 || zdy < L::FR) {  // uniform across the CTA: rows of a neighbouring sequence read as zero
          const uint4 z = make_uint4(0, 0, 0, 0);
          for (int idx = threadIdx.x; idx < zx * 16; idx += kCompThreads) {
            const int row = idx >> 4, part = idx & 15;
            *reinterpret_cast<uint4*>(stage_p + (part >> 3) * L::xbox + row * 128 + (part & 7) * 16) = z;
          }
          for (int idx = threadIdx.x; idx < (L::FR - zdy) * 16; idx += kCompThreads) {
            const int row = zdy + (idx >> 4), part = idx & 15;
            *reinterpret_cast<uint4*>(stage_p + L::x_bytes + (part >> 3) * L::dybox + row * 128 + (part & 7) * 16) = z;
          }
          comp_sync();
          if (zx > 0 && a.rm.halo != nullptr) {  // prefill with a cache: the cached tokens are the halo
            for (int idx = threadIdx.x; idx < (S - 1) * kBD5; idx += kCompThreads) {
              const int m = idx / kBD5 + 1, ch = idx - (m - 1) * kBD5;
              const int64_t row = ss - m - (r0 - kHalo5);
              const int64_t gch = ch_base + ch;
              if (row < 0 || row >= L::XR || gch >= a.D) continue;
              const int r = static_cast<int>(row), c64 = ch & 63;
              *reinterpret_cast<bf16*>(stage_p + (ch >> 6) * L::xbox + r * 128 + ((((c64 >> 3) ^ r) & 7) << 4) +
                                       (c64 & 7) * 2) = __float2bfloat16_rn(a.rm.halo_at(ss, ss - m, gch));
            }
            comp_sync();
          }
        }
      }

      // W_s fragments (C layout) at alpha rows ar..ar+15, from the basis fragments bw of tap s
      auto w_frag = [&](int ar, const uint32_t (&bw)[KT][4], float (&w)[2][4]) {
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
          uint32_t af[4];
          ldsm_x4(a_s + (ar & ~15) * ARB + alpha_off5<ARB>((ar & 15) + lrow, 2 * kt + lcol_chunk), af);
          if (kt == 0) {
            mma_bf16_z(w[0], af, bw[kt][0], bw[kt][1]);
            mma_bf16_z(w[1], af, bw[kt][2], bw[kt][3]);
          } else {
            mma_bf16(w[0], af, bw[kt][0], bw[kt][1]);
            mma_bf16(w[1], af, bw[kt][2], bw[kt][3]);
          }
        }
      };
      auto basis_frag = [&](int s, uint32_t (&bw)[KT][4]) {
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) ldsm_x4_t(basis_s + ((s * 2 + half) * KP + kt * 16) * 128 + row_sw, bw[kt]);
      };

      if constexpr (ACT) {
        // ---- dz = dy * silu'(pre) over tile rows 0..79 (the future rows feed dx), on chip
        if (valid) {
          for (int b = bp; b < 5; b += 2) {
            float pre[2][4] = {};
            if (16 * b < se - r0) {
#pragma unroll
              for (int s = 0; s < S; ++s) {
                const int j = S - 1 - s;
                uint32_t bw[KT][4];
                basis_frag(s, bw);
                float w[2][4];
                w_frag(16 * b, bw, w);
                const int rx = kHalo5 + 16 * b - j + lrow;
                uint32_t xr[4];
                ldsm_x4(x_s + x_box + rx * 128 + (((m_chunk ^ rx) & 7) << 4), xr);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                  ffma2(pre[nt][0], pre[nt][1], w[nt][0], w[nt][1], bf_lo(xr[2 * nt]), bf_hi(xr[2 * nt]));
                  ffma2(pre[nt][2], pre[nt][3], w[nt][2], w[nt][3], bf_lo(xr[2 * nt + 1]), bf_hi(xr[2 * nt + 1]));
                }
              }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int row = 16 * b + g + 8 * h;
                const int chunk = 2 * (cg & 3) + nt;
                uint32_t* d = reinterpret_cast<uint32_t*>(stage_p + L::x_bytes + half * L::dybox + row * 128 +
                                                          (((chunk ^ row) & 7) << 4) + 4 * q);
                const float2 ds = dsilu_bf2(pre[nt][2 * h], pre[nt][2 * h + 1]);
                const float2 o = __fmul2_rn(make_float2(bf_lo(*d), bf_hi(*d)), ds);
                *d = pack_bf16(o.x, o.y);
              }
          }
        }
        comp_sync();  // dz rows of the other warp of the channel group are read below
      }

      // dz of this warp's own blocks (the A operand rows of m)
      uint32_t dzo[2][4];
      float dxa[2][2][4];
#pragma unroll
      for (int bi = 0; bi < 2; ++bi) {
        ldsm_x4(x_s + dy_box + row_sw + (bp + 2 * bi) * 2048, dzo[bi]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) dxa[bi][nt][e] = 0.f;
      }

#pragma unroll
      for (int s = 0; s < S; ++s, ++ring_ctr) {
        const int slot = static_cast<int>(ring_ctr % L::NSLOT);
        const uint32_t use = ring_ctr / L::NSLOT;
        if (use > 0) wait_rec(bar_ring_empty + 8 * slot, (use - 1) & 1);
        if (valid) {
          const int j = S - 1 - s;
          const int rx = kHalo5 - j + lrow, ry = j + lrow;
          const uint32_t xo = x_s + x_box + static_cast<uint32_t>(rx * 128 + (((m_chunk ^ rx) & 7) << 4));
          const uint32_t yo = x_s + dy_box + static_cast<uint32_t>(ry * 128 + (((m_chunk ^ ry) & 7) << 4));
          const uint32_t ms = ring + slot * kSlotBytes + half * kSlotHalf + row_sw;
          uint32_t bw[KT][4];
          if (want_dx) basis_frag(s, bw);
#pragma unroll
          for (int bi = 0; bi < 2; ++bi) {
            const uint32_t b = static_cast<uint32_t>(bp + 2 * bi);
            if (want_dx) {
              float w[2][4];  // W_s at rows t + j
#pragma unroll
              for (int kt = 0; kt < KT; ++kt) {
                uint32_t af[4];
                ldsm_x4(a_s + b * 16 * ARB + alpha_off5<ARB>(ry, 2 * kt + lcol_chunk), af);
                if (kt == 0) {
                  mma_bf16_z(w[0], af, bw[kt][0], bw[kt][1]);
                  mma_bf16_z(w[1], af, bw[kt][2], bw[kt][3]);
                } else {
                  mma_bf16(w[0], af, bw[kt][0], bw[kt][1]);
                  mma_bf16(w[1], af, bw[kt][2], bw[kt][3]);
                }
              }
              uint32_t dys[4];
              ldsm_x4(yo + b * 2048, dys);
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                ffma2(dxa[bi][nt][0], dxa[bi][nt][1], w[nt][0], w[nt][1], bf_lo(dys[2 * nt]), bf_hi(dys[2 * nt]));
                ffma2(dxa[bi][nt][2], dxa[bi][nt][3], w[nt][2], w[nt][3], bf_lo(dys[2 * nt + 1]),
                      bf_hi(dys[2 * nt + 1]));
              }
            }
            uint32_t xr[4];
            ldsm_x4(xo + b * 2048, xr);
            // m = dz * x_shift rounded to bf16, into the slot (128-byte swizzled rows, as TMA writes them)
            stsm_x4(ms + b * 2048, hmul2_bf16(dzo[bi][0], xr[0]), hmul2_bf16(dzo[bi][1], xr[1]),
                    hmul2_bf16(dzo[bi][2], xr[2]), hmul2_bf16(dzo[bi][3], xr[3]));
          }
        }
        fence_proxy_async();  // the stmatrix writes, before the MMAs read the slot
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_ring_full + 8 * slot);
        if (warp < 4 && n >= kDaLag && s == (S > 1 ? 1 : 0)) drain_dalpha(n - kDaLag, prev_r0[n & 1], prev_rows[n & 1]);
      }

      if (valid && want_dx) {
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int b = bp + 2 * bi;
          bf16* dx_row = a.dx + (r0 + 16 * b + g) * a.D + ch_base + ch_w + 2 * q;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (16 * b + g + 8 * h < rows) {
#pragma unroll
              for (int nt = 0; nt < 2; ++nt)
                if (ch_base + ch_w + nt * 8 < a.D)
                  *reinterpret_cast<uint32_t*>(dx_row + 8 * h * a.D + nt * 8) =
                      pack_bf16(dxa[bi][nt][2 * h], dxa[bi][nt][2 * h + 1]);
            }
          }
        }
      }
      fence_proxy_async();  // this thread's writes to the stage, before TMA refills it
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_stage_empty + 8 * st);
      prev_r0[n & 1] = r0;
      prev_rows[n & 1] = rows;
    }
    if (warp < 4) {  // the items not yet read back: the last kDaLag
      const int n_it = static_cast<int>(i1 - i0);
      for (int n = std::max(0, n_it - kDaLag); n < n_it; ++n) drain_dalpha(n, prev_r0[n & 1], prev_rows[n & 1]);
    }

    // ---- the CTA's dbasis partial: db_part[group][k][s][ch]; TMEM lane = channel of the slice
    wait_rec(bar_db_done, 0);
    tc_fence_after5();
    const int quarter = warp & 3;
    const int64_t ch = ch_base + 32 * quarter + lane;
    const int64_t grp = blockIdx.y;
    for (int s = warp >> 2; s < S; s += 4) {
      uint32_t v[KP];
      if (any_valid) {
        tmem_ld_kp<KP>(tmem + (static_cast<uint32_t>(32 * quarter) << 16) + L::db_col + s * KP, v);
        tmem_ld_wait5();
      } else {
#pragma unroll
        for (int k = 0; k < KP; ++k) v[k] = 0u;
      }
      if (ch < a.D) {
#pragma unroll
        for (int k = 0; k < KP; ++k)
          if (k < a.K) a.db_part[((grp * a.K + k) * S + s) * a.D + ch] = __uint_as_float(v[k]);
      }
    }
  }

  griddep_launch_dependents();
  tc_fence_before5();
  __syncthreads();
  if (warp == kProdWarp) {
    tc_fence_after5();
    tmem_dealloc1(tmem, L::tmem_cols);
  }
}

// ------------------------------------------------------------------ host side

int sm_count5() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

struct Plan5 {
  RowMap rm;
  int64_t slices, groups, ipg;
};

// Token groups per slice.  One CTA runs per SM, so the grid runs in waves of sm_count CTAs,
// and a single wave of whole groups per slice can leave many SMs idle for the whole kernel
// (32 slices x 4 groups = 128 of 148 SMs).  The group count minimises
//   waves x (items per CTA + a CTA's fixed cost)
// where the fixed cost (basis staging, pipeline fill, the dbasis drain) is about one item;
// ties go to fewer groups (fewer dbasis partials).  At 32 slices x 512 items: 9 groups,
// two waves of 57 items (against one wave of 128).
Plan5 make_plan5(const moc_problem& p) {
  Plan5 pl;
  pl.rm = make_rowmap(p, kT5);
  pl.slices = ceil_div(p.dim, kBD5);
  const int64_t items = std::max<int64_t>(pl.rm.n_items(), 1);
  const int64_t sms = sm_count5();
  constexpr int64_t kCtaCost = 1;  // in items
  const int64_t g_max = std::min<int64_t>(items, std::max<int64_t>(1, 4 * sms / pl.slices));
  int64_t best_g = 1, best_cost = -1;
  for (int64_t g = 1; g <= g_max; ++g) {
    const int64_t ipg = ceil_div(items, g);
    const int64_t waves = ceil_div(pl.slices * ceil_div(items, ipg), sms);
    const int64_t cost = waves * (ipg + kCtaCost);
    if (best_cost < 0 || cost < best_cost) best_cost = cost, best_g = g;
  }
  pl.ipg = ceil_div(items, best_g);
  pl.groups = ceil_div(items, pl.ipg);
  return pl;
}

int configure5(const void* kern, bool (&configured)[64], int smem) {
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

template <int KT, int S, bool ACT>
int bwd5_inst(const moc_problem& p, Bwd5Args& args, const void* x, const void* alpha, const void* dy, void* dalpha,
              void* dbasis, cudaStream_t st) {
  using L = Layout5<KT, S, ACT>;
  const Plan5 pl = make_plan5(p);
  args.rm = pl.rm;
  args.items_per_group = pl.ipg;
  static bool configured[64] = {};
  int rc = configure5(reinterpret_cast<const void*>(k_bwd5<KT, S, ACT>), configured, L::total);
  if (rc != MOC_OK) return rc;
  const uint64_t D = static_cast<uint64_t>(p.dim), N = static_cast<uint64_t>(p.n_tokens);
  CUtensorMap xm, dym, am;
  rc = make_tmap_bf16_2d(&xm, x, D, N, D * 2, 64, L::XR, 128);
  if (rc == MOC_OK) rc = make_tmap_bf16_2d(&dym, dy, D, N, D * 2, 64, L::FR, 128);
  if (rc == MOC_OK)
    rc = make_tmap_bf16_2d(&am, alpha, static_cast<uint64_t>(p.n_bases), N, static_cast<uint64_t>(p.n_bases) * 2,
                           L::KP, L::AR, L::ARB);
  if (rc != MOC_OK) return rc;
  rc = note_cuda(launch_pdl(k_bwd5<KT, S, ACT>, dim3(static_cast<unsigned>(pl.slices), static_cast<unsigned>(pl.groups)),
                            dim3(kThreads5), L::total, st, xm, dym, am, args));
  note_launch();
  if (rc != MOC_OK) return rc;
  const int64_t nk = p.n_tokens * p.n_bases;
  const int64_t ksd = static_cast<int64_t>(p.n_bases) * p.kernel_size * p.dim;
  return tc_finalize(args.da_part, pl.slices, nk, dalpha, p.alpha_dtype, args.db_part, pl.groups, ksd, dbasis,
                     p.basis_dtype, st);
}

template <int S>
int bwd5_act(const moc_problem& p, Bwd5Args& args, const void* x, const void* alpha, const void* dy, void* da,
             void* db, cudaStream_t st) {
  return p.activation != 0 ? bwd5_inst<2, S, true>(p, args, x, alpha, dy, da, db, st)
                           : bwd5_inst<2, S, false>(p, args, x, alpha, dy, da, db, st);
}

void ws_split5(const moc_problem& p, size_t& da_bytes, size_t& db_bytes) {
  const Plan5 pl = make_plan5(p);
  da_bytes = align_up(static_cast<size_t>(pl.slices * p.n_tokens * p.n_bases) * sizeof(float), 256);
  db_bytes = align_up(static_cast<size_t>(pl.groups * p.n_bases * p.kernel_size * p.dim) * sizeof(float), 256);
}

bool aligned16_5(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

bool tc5_supported(const moc_problem& p) {
  return tc_conv_supported(p) && p.n_bases > 16 && p.kernel_size > 4;
}

size_t tc5_backward_ws(const moc_problem& p) {
  size_t da, db;
  ws_split5(p, da, db);
  return da + db;
}

int tc5_backward(const moc_problem& p, const void* x, const void* alpha, const void* basis, const void* dy, void* dx,
                 void* dalpha, void* dbasis, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!aligned16_5(x) || !aligned16_5(alpha) || !aligned16_5(basis) || !aligned16_5(dy) || (dx && !aligned16_5(dx)))
    return MOC_ERR_MISALIGNED;
  size_t da, db;
  ws_split5(p, da, db);
  if (ws_bytes < da + db) return MOC_ERR_WORKSPACE_TOO_SMALL;
  Bwd5Args args{};
  args.D = p.dim;
  args.K = p.n_bases;
  args.basis = static_cast<const bf16*>(basis);
  args.dx = static_cast<bf16*>(dx);
  args.da_part = static_cast<float*>(ws);
  args.db_part = reinterpret_cast<float*>(static_cast<char*>(ws) + da);
  args.n_tokens = p.n_tokens;
  switch (p.kernel_size) {
    case 5: return bwd5_act<5>(p, args, x, alpha, dy, dalpha, dbasis, st);
    case 6: return bwd5_act<6>(p, args, x, alpha, dy, dalpha, dbasis, st);
    case 7: return bwd5_act<7>(p, args, x, alpha, dy, dalpha, dbasis, st);
    case 8: return bwd5_act<8>(p, args, x, alpha, dy, dalpha, dbasis, st);
    default: return MOC_ERR_UNSUPPORTED_SHAPE;
  }
}

int bwd5_status(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_bwd5_status, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_bwd5_status, &zero, sizeof(int));
    if (e != cudaSuccess) return note_cuda(e);
  }
  *out = v;
  return MOC_OK;
}

}  // namespace moc
