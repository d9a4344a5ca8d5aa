// Gradient all-reduce over NVLink peer memory for the data-parallel MoC step.
//
// The one collective of the data-parallel step is a sum over ranks of the parameter
// gradients (conv_bases [K, S, D] and router [K, Dz]: 640 KiB of fp32 at config 2), small
// enough that its cost is latency.  Every rank owns an exchange buffer in its own HBM,
// opened by every other rank through CUDA IPC (peer pointers over NVLink / NVSwitch).  One
// kernel per call:
//   1. CTA c converts its slice of the gradients to fp32 into this rank's buffer (one of two
//      halves, alternating per call so that a slow peer's reads of the previous call's half
//      never race with this call's writes);
//   2. it publishes the slice: its call counter, stored with system-scope release
//      semantics into slot (c, rank) of every rank's flag array;
//   3. it waits, with a poll limit, until slot (c, r) of its own flag array holds the call
//      counter for every rank r;
//   4. it adds the slice of every rank's buffer in rank order (the same fp32 sum on every
//      rank, so the replicas stay bitwise identical) and writes it back in the gradient dtype.
// CTAs only wait for the same CTA index on other GPUs, the grid is one wave, and the call
// counter lives in device memory (CTA c keeps its own), so the launch can be captured in a
// CUDA graph and replayed.  A wait that runs out (after the communicator's poll limit)
// records MOC_STATUS_WAIT_TIMEOUT in the communicator's status word and the library's, and
// the CTA leaves its gradients unchanged.  After a timeout the ranks' call counters no
// longer pair up (the timed-out call advanced them on some ranks only); comm_reset zeroes
// this rank's counters, flags and status, and once every rank has reset, with no call in
// flight anywhere, the next call pairs again.
#include <algorithm>
#include <cstring>

#include "moc_common.cuh"
#include "moc_internal.h"
#include "moc_tma.cuh"

namespace moc {

__device__ int g_comm_status;

namespace {

constexpr int kCommCtas = 128;
constexpr int kCommThreads = 256;
constexpr uint32_t kCommPollLimit = 1u << 22;

struct CommSeg {
  void* data;
  int64_t n;
  int dtype;
};

struct CommArgs {
  float* bufs[MOC_COMM_MAX_RANKS];        // every rank's exchange buffer (two halves of `cap` floats)
  uint32_t* flags[MOC_COMM_MAX_RANKS];    // every rank's flag array [kCommCtas][world]
  uint32_t* counter;                      // this rank's per-CTA call counters [kCommCtas]
  int* status;                            // this communicator's status word
  uint32_t poll_limit;                    // polls of a peer's flag before giving up
  CommSeg seg[MOC_COMM_MAX_SEGMENTS];
  int n_seg;
  int64_t total, cap;
  int rank, world;
};

__device__ __forceinline__ float seg_load(const CommSeg& s, int64_t i) { return ld_any(s.data, s.dtype, i); }
__device__ __forceinline__ void seg_store(const CommSeg& s, int64_t i, float v) { st_any(s.data, s.dtype, i, v); }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// element i of the concatenated segments
template <class F>
__device__ __forceinline__ void for_seg(const CommArgs& a, int64_t i, F f) {
  int64_t base = 0;
#pragma unroll
  for (int s = 0; s < MOC_COMM_MAX_SEGMENTS; ++s) {
    if (s < a.n_seg && i >= base && i < base + a.seg[s].n) {
      f(a.seg[s], i - base);
      return;
    }
    base += s < a.n_seg ? a.seg[s].n : 0;
  }
}

__global__ void __launch_bounds__(kCommThreads) k_allreduce(const __grid_constant__ CommArgs a) {
  __shared__ uint32_t call;
  __shared__ int ok;
  const int c = blockIdx.x;
  const int64_t per = (a.total + kCommCtas - 1) / kCommCtas;
  const int64_t i0 = c * per, i1 = i0 + per < a.total ? i0 + per : a.total;
  if (threadIdx.x == 0) call = a.counter[c] + 1;
  __syncthreads();
  const uint32_t step = call;
  const int64_t half = static_cast<int64_t>(step & 1) * a.cap;
  float* mine = a.bufs[a.rank] + half;

  // 1. this rank's slice, as fp32, into its own buffer; each thread loads a batch of
  // elements before it stores any (the compiler cannot tell the gradients from the buffer)
  constexpr int kBatch = 8;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += kBatch * kCommThreads) {
    float v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t e = i + u * kCommThreads;
      v[u] = 0.f;
      if (e < i1) for_seg(a, e, [&](const CommSeg& sg, int64_t j) { v[u] = seg_load(sg, j); });
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (i + u * kCommThreads < i1) mine[i + u * kCommThreads] = v[u];
  }
  __syncthreads();
  // 2. publish it to every rank (the release store orders the CTA's slice before the flag)
  if (threadIdx.x < a.world) st_release_sys(a.flags[threadIdx.x] + c * a.world + a.rank, step);
  // 3. wait for every rank's slice
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint32_t* f = a.flags[a.rank] + c * a.world + threadIdx.x;
    uint32_t n = 0;
    while (static_cast<int32_t>(ld_acquire_sys(f) - step) < 0) {
      if (++n >= a.poll_limit) {
        ok = 0;
        atomicOr(&g_comm_status, kStatusWaitTimeout);
        atomicOr(a.status, kStatusWaitTimeout);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  // 4. the rank-ordered sum of every rank's slice: the batch's loads from all ranks are in
  // flight at once (one NVLink round trip, not one per rank), then added in rank order
  if (ok) {
    for (int64_t i = i0 + threadIdx.x; i < i1; i += kBatch * kCommThreads) {
      float t[MOC_COMM_MAX_RANKS][kBatch];
#pragma unroll
      for (int r = 0; r < MOC_COMM_MAX_RANKS; ++r) {
        if (r < a.world) {
          const float* src = a.bufs[r] + half;
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int64_t e = i + u * kCommThreads;
            t[r][u] = e < i1 ? __ldcg(src + e) : 0.f;  // L2 / peer, never a stale L1 line
          }
        }
      }
      float v[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) v[u] = 0.f;
#pragma unroll
      for (int r = 0; r < MOC_COMM_MAX_RANKS; ++r)
        if (r < a.world) {
#pragma unroll
          for (int u = 0; u < kBatch; ++u) v[u] += t[r][u];
        }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t e = i + u * kCommThreads;
        if (e < i1) for_seg(a, e, [&](const CommSeg& sg, int64_t j) { seg_store(sg, j, v[u]); });
      }
    }
  }
  if (threadIdx.x == 0) a.counter[c] = step;
}

}  // namespace

struct CommImpl {
  int rank = 0, world = 0, device = -1;
  int64_t cap = 0;          // floats per buffer half
  uint32_t poll_limit = kCommPollLimit;
  char* local = nullptr;    // this rank's allocation: [2 * cap floats | flags | counters | status]
  size_t local_bytes = 0;
  char* peers[MOC_COMM_MAX_RANKS] = {};  // opened IPC mappings (peers[rank] = local)
};

// Byte offsets inside a rank's allocation; flags, counters and the status word are one
// contiguous tail [flags_off, total), which comm_reset clears.
static size_t comm_layout(int64_t cap, int world, size_t* flags_off, size_t* counter_off, size_t* status_off) {
  *flags_off = align_up(static_cast<size_t>(2 * cap) * sizeof(float), 256);
  *counter_off = align_up(*flags_off + static_cast<size_t>(kCommCtas) * world * sizeof(uint32_t), 256);
  *status_off = align_up(*counter_off + kCommCtas * sizeof(uint32_t), 256);
  return align_up(*status_off + sizeof(int), 256);
}

int comm_create(int rank, int world, int64_t capacity, CommImpl** out, void* handle_out) {
  CommImpl* c = new CommImpl();
  c->rank = rank;
  c->world = world;
  c->cap = capacity;
  cudaError_t e = cudaGetDevice(&c->device);
  size_t foff, coff, soff;
  c->local_bytes = comm_layout(capacity, world, &foff, &coff, &soff);
  if (e == cudaSuccess) e = cudaMalloc(&c->local, c->local_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->local_bytes);
  cudaIpcMemHandle_t h{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return note_cuda(e);
  }
  std::memcpy(handle_out, &h, sizeof(h));
  c->peers[rank] = c->local;
  *out = c;
  return MOC_OK;
}

int comm_connect(CommImpl* c, const void* handles) {
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + r * MOC_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return note_cuda(e);
    c->peers[r] = static_cast<char*>(p);
  }
  return MOC_OK;
}

int comm_allreduce(CommImpl* c, int n_seg, void* const* data, const int64_t* n, const int32_t* dtype,
                   cudaStream_t st) {
  CommArgs a{};
  size_t foff, coff, soff;
  comm_layout(c->cap, c->world, &foff, &coff, &soff);
  for (int r = 0; r < c->world; ++r) {
    if (c->peers[r] == nullptr) return MOC_ERR_INVALID_ARGUMENT;  // not connected
    a.bufs[r] = reinterpret_cast<float*>(c->peers[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(c->peers[r] + foff);
  }
  a.counter = reinterpret_cast<uint32_t*>(c->local + coff);
  a.status = reinterpret_cast<int*>(c->local + soff);
  a.poll_limit = c->poll_limit;
  a.n_seg = n_seg;
  a.total = 0;
  for (int s = 0; s < n_seg; ++s) {
    a.seg[s] = CommSeg{data[s], n[s], dtype[s]};
    a.total += n[s];
  }
  if (a.total > c->cap) return MOC_ERR_SCRATCH_LIMIT;
  a.cap = c->cap;
  a.rank = c->rank;
  a.world = c->world;
  if (a.total == 0) return MOC_OK;
  k_allreduce<<<kCommCtas, kCommThreads, 0, st>>>(a);
  note_launch();
  return note_cuda(cudaGetLastError());
}

int comm_destroy(CommImpl* c) {
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < c->world; ++r) {
    if (r != c->rank && c->peers[r] != nullptr) {
      const cudaError_t e = cudaIpcCloseMemHandle(c->peers[r]);
      if (first == cudaSuccess) first = e;
    }
  }
  if (c->local) {
    const cudaError_t e = cudaFree(c->local);
    if (first == cudaSuccess) first = e;
  }
  delete c;
  return note_cuda(first);
}

void comm_set_poll_limit(CommImpl* c, uint32_t limit) { c->poll_limit = limit > 0 ? limit : kCommPollLimit; }

int comm_reset(CommImpl* c, cudaStream_t st) {
  size_t foff, coff, soff;
  const size_t total = comm_layout(c->cap, c->world, &foff, &coff, &soff);
  return note_cuda(cudaMemsetAsync(c->local + foff, 0, total - foff, st));
}

int comm_own_status(CommImpl* c, int* out, bool clear) {
  size_t foff, coff, soff;
  comm_layout(c->cap, c->world, &foff, &coff, &soff);
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, c->local + soff, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && v != 0) e = cudaMemset(c->local + soff, 0, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  *out = v;
  return MOC_OK;
}

// Probe of the timeout path: the all-reduce kernel, as rank 0 of a world of two whose
// rank 1 never calls.  Both ranks' buffers and flag arrays are one fixed local array, so
// rank 1's flags stay zero; every CTA waits `limit` polls, records the timeout and leaves
// the probe data unchanged.
__device__ float g_probe_buf[3 * 128];
__device__ uint32_t g_probe_flags[kCommCtas * 2 + kCommCtas];
__device__ int g_probe_status;

int comm_wait_timeout_probe(uint32_t limit, cudaStream_t st) {
  void *buf = nullptr, *flags = nullptr, *status = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&buf, g_probe_buf);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&flags, g_probe_flags);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&status, g_probe_status);
  if (e == cudaSuccess) e = cudaMemsetAsync(flags, 0, sizeof(g_probe_flags), st);
  if (e != cudaSuccess) return note_cuda(e);
  CommArgs a{};
  float* data = static_cast<float*>(buf) + 256;  // the "gradient": 128 floats after the two exchange halves
  a.bufs[0] = a.bufs[1] = static_cast<float*>(buf);
  a.flags[0] = a.flags[1] = static_cast<uint32_t*>(flags);
  a.counter = static_cast<uint32_t*>(flags) + kCommCtas * 2;
  a.status = static_cast<int*>(status);
  a.poll_limit = limit > 0 ? limit : 1;
  a.n_seg = 1;
  a.seg[0] = CommSeg{data, 128, MOC_DTYPE_F32};
  a.total = 128;
  a.cap = 128;  // the exchange halves are buf[0, 128) and buf[128, 256)
  a.rank = 0;
  a.world = 2;
  k_allreduce<<<kCommCtas, kCommThreads, 0, st>>>(a);
  note_launch();
  return note_cuda(cudaGetLastError());
}

int comm_status(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_comm_status, sizeof(int));
  if (e != cudaSuccess) return note_cuda(e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_comm_status, &zero, sizeof(int));
    if (e != cudaSuccess) return note_cuda(e);
  }
  *out = v;
  return MOC_OK;
}

}  // namespace moc
