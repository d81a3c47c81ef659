// Expert-parallel exchange of the MoE block over peer memory (NVLink / NVSwitch).
//
// The reference runs every expert of a layer on one device
// (parrot/model.py:521-551); here G ranks, one process per GPU, each hold
// their own tokens and a set of expert slots.  Each source's plan names the
// rank that computes its rows of each expert: one owner per expert, except
// that an expert every rank holds (a replicated, heavily routed one) is
// computed by each source on its own rows.  Every
// rank owns one "EP buffer" that the other ranks map into their address space
// (CUDA IPC).  One MoE call moves data only by stores into those buffers:
//
//   send     the dispatched rows (packed destination-major by the grouping
//            kernel) are stored into each destination's receive region for
//            this source, with this rank's per-local-expert counts and the
//            offset of those rows in its own dispatch order; then one arrival
//            flag per destination;
//   receive  waits for every source's arrival flag and turns the counts into
//            the expert GEMM's segment table (one segment per (source, local
//            expert slot)) on the device;
//   return   the expert outputs are stored back into each source's return
//            region at the offsets the source sent, then one flag per source;
//   combine  (route.cu) waits for every expert rank's return flag, then adds
//            the weighted outputs to the shared expert's in expert-id order.
//
// The row copies of send and return can also be left to the kernels that
// produce the rows: the grouping kernel (route.cu) stores each dispatched
// row into its destination's receive region, the down GEMM's epilogue
// (gemm.cu) each output into its source's return region, and both fence at
// system scope before they complete; send and return then run as one block
// that writes the counts and raises the flags (rows_sent).
//
// No host synchronisation and no size known only on the device reaches the
// host, so the layer can be captured in a CUDA graph.  Flags carry an epoch
// (the number of sends this rank has made, kept in its own buffer); every
// rank makes the same calls, so a rank waits for flag >= its own epoch.  A
// buffer region is only rewritten after its reader has provably finished
// with it: a source sends call i + 1 only after its combine of call i, which
// waited for every expert rank's return of call i, which each expert rank
// issued after its GEMM of call i had read its receive regions.
//
// Every wait is bounded (wait_ns): on timeout the kernel records
// kStatusWaitTimeout in the EP buffer's status word, treats the missing
// source as sending nothing and returns.  No TMA, no multicast: peer memory
// is touched only by 16-byte stores and flag loads/stores.
#include "kernels.h"
#include "peer.cuh"

namespace parrot {

namespace {

// Rows a warp moves per batch: every load of the batch is issued before its
// stores, so a lane keeps up to kRowBatch * 4 16-byte loads in flight.
constexpr int kRowBatch = 4;

// One warp copies rows [first, first + n), n <= kRowBatch, of nvec 16-byte
// vectors each (nvec <= 128): row k goes from src(k) to dst(k).
template <typename Src, typename Dst>
__device__ __forceinline__ void copy_rows(int first, int n, int nvec, int lane, Src src, Dst dst) {
  uint4 v[kRowBatch][4];
#pragma unroll
  for (int k = 0; k < kRowBatch; ++k) {
    if (k < n) {
      const uint4* s = src(first + k);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (lane + 32 * c < nvec) v[k][c] = __ldcg(s + lane + 32 * c);
    }
  }
#pragma unroll
  for (int k = 0; k < kRowBatch; ++k) {
    if (k < n) {
      uint4* d = dst(first + k);
      if (d == nullptr) continue;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (lane + 32 * c < nvec) d[lane + 32 * c] = v[k][c];
    }
  }
}

// Last-CTA election after every CTA's stores: each CTA fences its stores at
// system scope, then counts itself; the CTA that counts last resets the
// counter and returns true.
__device__ bool last_cta(unsigned* counter) {
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
    if (last) *counter = 0;
  }
  __syncthreads();
  return last;
}

}  // namespace

__global__ void __launch_bounds__(256) ep_send_kernel(EpSendArgs a) {
  __shared__ int n_s[kEpMaxRanks], base_s[kEpMaxRanks];
  griddep_wait();
  griddep_launch();
  const int G = a.ranks;
  if (threadIdx.x < G) {
    const int q = threadIdx.x;
    int n = 0;
    if (a.tokens > 0)
      for (int j = 0; j < kMaxExperts; ++j)
        if (a.plan[q][j] >= 0) n += a.counts[a.plan[q][j]];
    n_s[q] = n;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // the packed rows are destination-major from row 0
    int at = 0;
    for (int q = 0; q < G; ++q) {
      base_s[q] = at;
      at += n_s[q];
    }
  }
  __syncthreads();
  const int nvec = a.dim >> 3;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int total = a.rows_sent ? 0 : 2 * a.tokens;
  const size_t region = (size_t)2 * a.max_tokens;
  const uint4* rows = reinterpret_cast<const uint4*>(a.rows);
  for (int i = (blockIdx.x * warps + (threadIdx.x >> 5)) * kRowBatch; i < total;
       i += gridDim.x * warps * kRowBatch) {
    copy_rows(
        i, min(kRowBatch, total - i), nvec, lane,
        [&](int r) { return rows + (size_t)r * nvec; },
        [&](int r) -> uint4* {
          int q = 0;
          while (q + 1 < G && r >= base_s[q] + n_s[q]) ++q;
          const int k = r - base_s[q];
          if (k < 0 || k >= n_s[q] || k >= (int)region) {
            if (lane == 0) report_status(a.status, kStatusBadIndex, 20, r);
            return nullptr;
          }
          return reinterpret_cast<uint4*>(a.peers[q] + a.off_recv) +
                 ((size_t)a.rank * region + k) * nvec;
        });
  }
  if (!last_cta(a.counter)) return;
  const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1;
  if (threadIdx.x < G) {
    const int q = threadIdx.x;
    int* meta = reinterpret_cast<int*>(a.peers[q] + a.off_meta) + a.rank * kEpMetaStride;
    for (int j = 0; j < kMaxExperts; ++j)
      meta[j] = (a.tokens > 0 && a.plan[q][j] >= 0) ? a.counts[a.plan[q][j]] : 0;
    meta[kEpMetaStride - 1] = base_s[q];
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned*>(a.peers[q] + a.off_flags_in) + a.rank, e);
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.epoch = e;
}

__global__ void __launch_bounds__(32) ep_receive_kernel(EpReceiveArgs a) {
  __shared__ int n_s[kEpMaxRanks][kMaxExperts];
  griddep_wait();
  griddep_launch();
  const int G = a.ranks, El = a.slots;
  const unsigned e = *reinterpret_cast<const volatile unsigned*>(a.epoch);
  const int region = 2 * a.max_tokens;
  if (threadIdx.x < G) {
    const int s = threadIdx.x;
    bool ok = wait_flag(a.flags_in + s, e, a.wait_ns, a.status);
    if (!ok) report_status(a.status, kStatusWaitTimeout, 21, s);
    const int* meta = a.meta + s * kEpMetaStride;
    int total = 0;
    for (int j = 0; j < El; ++j) {
      const int n = ok ? ld_volatile(meta + j) : 0;
      n_s[s][j] = n;
      if (n < 0) ok = false;
      total += n;
    }
    int back = ok ? ld_volatile(meta + kEpMetaStride - 1) : 0;
    if (ok && (total > region || back < 0 || back + total > region)) {
      report_status(a.status, kStatusBadShape, 22, s);
      ok = false;
    }
    if (!ok) {
      for (int j = 0; j < El; ++j) n_s[s][j] = 0;
      total = 0;
      back = 0;
    }
    a.back_n[s] = total;
    a.back_base[s] = back;
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    for (int s = 0; s < G; ++s) {
      int at = s * region;
      for (int j = 0; j < El; ++j) {
        const int g = s * El + j;
        a.seg_rows[g] = n_s[s][j];
        a.seg_base[g] = at;
        a.seg_expert[g] = j;
        at += n_s[s][j];
      }
    }
  }
}

__global__ void __launch_bounds__(256) ep_return_kernel(EpReturnArgs a) {
  __shared__ int n_s[kEpMaxRanks], start_s[kEpMaxRanks + 1], base_s[kEpMaxRanks];
  griddep_wait();
  griddep_launch();
  const int G = a.ranks;
  if (threadIdx.x == 0) {
    int at = 0;
    for (int s = 0; s < G; ++s) {
      n_s[s] = a.back_n[s];
      base_s[s] = a.back_base[s];
      start_s[s] = at;
      at += n_s[s];
    }
    start_s[G] = at;
  }
  __syncthreads();
  const int nvec = a.dim >> 3;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const size_t region = (size_t)2 * a.max_tokens;
  const uint4* y = reinterpret_cast<const uint4*>(a.y);
  const int total = a.rows_sent ? 0 : start_s[G];
  auto source_of = [&](int r) {
    int s = 0;
    while (s + 1 < G && r >= start_s[s + 1]) ++s;
    return s;
  };
  for (int i = (blockIdx.x * warps + (threadIdx.x >> 5)) * kRowBatch; i < total;
       i += gridDim.x * warps * kRowBatch) {
    copy_rows(
        i, min(kRowBatch, total - i), nvec, lane,
        [&](int r) {
          const int s = source_of(r);
          return y + ((size_t)s * region + (r - start_s[s])) * nvec;
        },
        [&](int r) -> uint4* {
          const int s = source_of(r);
          return reinterpret_cast<uint4*>(a.peers[s] + a.off_back) +
                 (size_t)(base_s[s] + r - start_s[s]) * nvec;
        });
  }
  if (!last_cta(a.counter)) return;
  const unsigned e = *reinterpret_cast<const volatile unsigned*>(a.epoch);
  if (threadIdx.x < G) {
    const int s = threadIdx.x;
    st_release_sys(reinterpret_cast<unsigned*>(a.peers[s] + a.off_flags_back) + a.rank, e);
  }
}

int launch_ep_send(const EpSendArgs& a, int sms, cudaStream_t stream) {
  const int rows = a.rows_sent ? 0 : 2 * a.tokens;
  int grid = (rows + 8 * kRowBatch - 1) / (8 * kRowBatch);
  if (grid > 2 * sms) grid = 2 * sms;
  if (grid < 1) grid = 1;
  return launch_pdl(ep_send_kernel, dim3(grid), dim3(256), 0, stream, a) == cudaSuccess ? 0 : -1;
}

int launch_ep_receive(const EpReceiveArgs& a, cudaStream_t stream) {
  return launch_pdl(ep_receive_kernel, dim3(1), dim3(32), 0, stream, a) == cudaSuccess ? 0 : -1;
}

int launch_ep_return(const EpReturnArgs& a, int sms, cudaStream_t stream) {
  // the row count is only known on the device: a fixed grid strides over it
  return launch_pdl(ep_return_kernel, dim3(a.rows_sent ? 1 : 2 * sms), dim3(256), 0, stream, a) ==
                 cudaSuccess
             ? 0
             : -1;
}

}  // namespace parrot
