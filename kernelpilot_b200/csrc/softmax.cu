// Row softmax over the last dimension of a contiguous (M, N) matrix (kp.softmax).
//
// Replaces kernelpilot's csrc/kernels/softmax.hip (stages :14-113, dispatch
// :116-152). The contract is the same (fp32 math, output in the input dtype,
// empty input is a no-op); the B200 kernel is new:
//
//   variant 0  thread per row, three passes over global memory (baseline)
//   variant 1  CTA per row, three coalesced passes with block reductions
//   variant 2  "staged": a persistent grid; each CTA owns a ring of row buffers in
//              shared memory filled by 1-D bulk (TMA) copies issued `stages` rows
//              ahead, so HBM reads of later rows overlap the reductions of the
//              current one. Every thread keeps its slice of the row in registers:
//              max -> exp2 -> sum -> scale -> 128-bit streaming stores. HBM sees one
//              read and one write per element. The arithmetic is packed (3-input max,
//              f32x2 FMA/add/mul) and exp2 runs on the MUFU directly, about 4.5
//              instructions per element, so the kernel stays memory-bound.
//              Rows longer than 1024 threads x 24 (fp32) / 32 (16-bit) values are
//              split over a thread-block cluster of 2, 4 or 8 CTAs ("cluster"): each
//              CTA runs the same ring on its slice of the row and the row's max and
//              sum are merged through distributed shared memory, so such rows still
//              cost one HBM read and one write. Rows beyond 8 CTAs' registers
//              (196,608 fp32 / 262,144 16-bit values) take "two-pass": online
//              (max, sum) in one read, normalise in a second.
//
// Rows need not start on a 16-byte boundary (fp32 N=4097 rows are 16388 bytes):
// each row is viewed through the aligned window that contains it. Whole 16-byte
// vectors inside the row are moved as vectors; the partial vectors at each end of a
// row use masked scalar accesses, and the bulk copy never reaches outside x. When
// every row is aligned (kAligned) the masking disappears from the kernel.
#include <algorithm>

#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxStages = 8;
// 16-byte vectors per thread in the staged kernel: at most 24 (fp32) or 32 (16-bit)
// row values live in registers, which keeps 1024-thread CTAs free of spills.
template <typename T> constexpr int staged_max_v() { return sizeof(T) == 4 ? 6 : 4; }

// ------------------------------------------------------------------ variant 0

template <typename T>
__global__ void softmax_thread_row(const T* __restrict__ x, T* __restrict__ y, int64_t M,
                                   int64_t N) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= M) return;
  const T* xr = x + row * N;
  T* yr = y + row * N;
  float m = -INFINITY;
  for (int64_t j = 0; j < N; ++j) m = fmaxf(m, to_f(xr[j]));
  const float ml = m * kLog2e;
  float d = 0.f;
  for (int64_t j = 0; j < N; ++j) d += exp2f(fmaf(to_f(xr[j]), kLog2e, -ml));
  const float inv = 1.f / d;
  for (int64_t j = 0; j < N; ++j) yr[j] = from_f<T>(exp2f(fmaf(to_f(xr[j]), kLog2e, -ml)) * inv);
}

// ------------------------------------------------------------------ variant 1

template <typename T>
__global__ void __launch_bounds__(256) softmax_block_row(const T* __restrict__ x,
                                                         T* __restrict__ y, int64_t N) {
  __shared__ float s_max[kWarp], s_sum[kWarp];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * N;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * N;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) m = fmaxf(m, to_f(xr[j]));
  m = block_reduce<true>(m, s_max);
  const float ml = m * kLog2e;
  float d = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
    d += exp2f(fmaf(to_f(xr[j]), kLog2e, -ml));
  d = block_reduce<false>(d, s_sum);
  const float inv = 1.f / d;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
    yr[j] = from_f<T>(exp2f(fmaf(to_f(xr[j]), kLog2e, -ml)) * inv);
}

// ------------------------------------------------------------------ variant 2: staged

// Geometry of one row seen through its aligned window.
struct RowView {
  uintptr_t win;    // 16-byte aligned address at or below the row start
  int a;            // elements between `win` and the row start
  int nv;           // 16-byte vectors covering the row
};

template <typename T>
__device__ __forceinline__ RowView row_view(uintptr_t row_start, int N) {
  constexpr int VN = Vec<T>::kN;
  RowView r;
  r.win = row_start & ~uintptr_t(15);
  r.a = static_cast<int>((row_start - r.win) / sizeof(T));
  r.nv = (r.a + N + VN - 1) / VN;
  return r;
}

// Per-vector element math on registers, two lanes at a time.
template <int VN>
__device__ __forceinline__ float vmax(const float (&f)[VN], float m) {
#pragma unroll
  for (int l = 0; l < VN; l += 2) m = max3f(m, f[l], f[l + 1]);
  return m;
}

// f <- exp2(f * log2e - ml); returns the running sum of the new values (two partials).
template <int VN>
__device__ __forceinline__ float2 vexp(float (&f)[VN], float2 acc, float neg_ml) {
  const float2 s2 = make_float2(kLog2e, kLog2e), c2 = make_float2(neg_ml, neg_ml);
#pragma unroll
  for (int l = 0; l < VN; l += 2) {
    float2 t = __ffma2_rn(make_float2(f[l], f[l + 1]), s2, c2);
    t.x = ex2f(t.x);
    t.y = ex2f(t.y);
    f[l] = t.x;
    f[l + 1] = t.y;
    acc = __fadd2_rn(acc, t);
  }
  return acc;
}

template <int VN>
__device__ __forceinline__ void vscale(float (&f)[VN], float inv) {
  const float2 i2 = make_float2(inv, inv);
#pragma unroll
  for (int l = 0; l < VN; l += 2) {
    const float2 t = __fmul2_rn(make_float2(f[l], f[l + 1]), i2);
    f[l] = t.x;
    f[l + 1] = t.y;
  }
}

// ---- row statistics with one block barrier
//
// Each warp takes the max of its values, exponentiates them against it (in log2
// units: f <- 2^(x*log2e - ml_w)) and sums them; lane 0 posts (ml_w, d_w) for its
// warp, with d_w = -1 when the warp's copy wait gave up. After ONE barrier every warp
// merges the posted pairs the same way (lane i takes warp i's pair; a shuffle max and
// a shuffle sum of d_i * 2^(ml_i - ML)), so all warps get the same (ML, D) bits, and a
// value's softmax is f * 2^(ml_w - ML) / D. The posts alternate between two buffers
// by row parity: a warp writes row r+2's post only after the barrier of row r+1,
// which every warp reaches after reading row r's posts.
struct RowStats {
  float ml_warp;  // this warp's max (log2 units)
  float ml;       // the block's max (log2 units)
  float d;        // the block's sum of 2^(x*log2e - ml)
  bool ok;        // no warp's copy wait gave up
};

template <int V, int VN>
__device__ __forceinline__ RowStats block_row_stats(float (&f)[V][VN], bool ok, float2* post) {
  const int lane = threadIdx.x & (kWarp - 1), wid = threadIdx.x / kWarp;
  const int nwarps = blockDim.x / kWarp;
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < V; ++k) mx = vmax<VN>(f[k], mx);
  mx = warp_max(mx);
  RowStats r;
  r.ml_warp = mx * kLog2e;
  const float neg = r.ml_warp == -INFINITY ? 0.f : -r.ml_warp;
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < V; ++k) acc = vexp<VN>(f[k], acc, neg);
  const float d = warp_sum(acc.x + acc.y);
  const bool wok = __all_sync(kFull, ok);
  if (lane == 0) post[wid] = make_float2(r.ml_warp, wok ? d : -1.f);
  __syncthreads();
  const float2 pw = lane < nwarps ? post[lane] : make_float2(-INFINITY, 0.f);
  r.ok = !__any_sync(kFull, pw.y < 0.f);
  r.ml = warp_max(pw.x);
  const float term = pw.x == -INFINITY ? 0.f : pw.y * ex2f(pw.x - r.ml);
  r.d = warp_sum(term);
  return r;
}

// factor that turns this warp's 2^(x*log2e - ml_warp) into softmax values, given the
// row's max ml and sum d (both in the same units)
__device__ __forceinline__ float warp_scale(float ml_warp, float ml, float d) {
  return ml_warp == -INFINITY ? 0.f : ex2f(ml_warp - ml) / d;
}

template <typename T, int V, bool kAligned>
__global__ void __launch_bounds__(1024)
softmax_staged(const T* __restrict__ x, T* __restrict__ y, int64_t M, int N, int stages,
               uint32_t stage_bytes, unsigned* err) {
  constexpr int VN = Vec<T>::kN;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint8_t* ring = smem + 128;
  __shared__ float2 post[2][kWarp];

  const uintptr_t xbase = reinterpret_cast<uintptr_t>(x);
  const uintptr_t xend = xbase + static_cast<uintptr_t>(M) * N * sizeof(T);
  const uintptr_t ok_lo = (xbase + 15) & ~uintptr_t(15);  // bulk copies stay in [ok_lo, ok_hi)
  const uintptr_t ok_hi = xend & ~uintptr_t(15);
  const size_t row_bytes = static_cast<size_t>(N) * sizeof(T);
  const bool y_vec = ((reinterpret_cast<uintptr_t>(y) ^ xbase) & 15) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t policy = l2_evict_first_policy();

  // copied part of a row's window, in vectors: [vlo, vhi)
  auto copy_span = [&](const RowView& rv, int& vlo, int& vhi) {
    const uintptr_t cs = rv.win > ok_lo ? rv.win : ok_lo;
    const uintptr_t we = rv.win + static_cast<uintptr_t>(rv.nv) * 16;
    const uintptr_t ce = we < ok_hi ? we : ok_hi;
    vlo = static_cast<int>((cs - rv.win) / 16);
    vhi = ce > cs ? static_cast<int>((ce - rv.win) / 16) : vlo;
  };

  // Thread 0: start the copy of `row` into ring slot `slot`.
  auto issue = [&](int64_t row, int slot) {
    const RowView rv = row_view<T>(xbase + static_cast<uintptr_t>(row) * row_bytes, N);
    int vlo, vhi;
    copy_span(rv, vlo, vhi);
    if (vhi > vlo) {
      const uint32_t bytes = static_cast<uint32_t>(vhi - vlo) * 16;
      mbar_arrive_expect_tx(&full[slot], bytes);
      bulk_g2s(ring + size_t(slot) * stage_bytes + vlo * 16,
               reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(vlo) * 16), bytes,
               &full[slot], policy);
    } else {
      mbar_arrive(&full[slot]);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      const int64_t r = blockIdx.x + static_cast<int64_t>(s) * gridDim.x;
      if (r < M) issue(r, s);
    }
  }

  int it = 0;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x, ++it) {
    const int slot = it % stages;
    const bool ok = mbar_wait(&full[slot], static_cast<uint32_t>((it / stages) & 1), err);

    const RowView rv = row_view<T>(xbase + static_cast<uintptr_t>(row) * row_bytes, N);
    int vlo = 0, vhi = rv.nv;
    if (!kAligned) copy_span(rv, vlo, vhi);
    const uint8_t* stage = ring + size_t(slot) * stage_bytes;
    const T* xr = x + row * N;

    float f[V][VN];
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = threadIdx.x + k * blockDim.x;
      if (kAligned) {
        if (j < rv.nv) {
          unpack<T>(*reinterpret_cast<const uint4*>(stage + j * 16), f[k]);
        } else {
#pragma unroll
          for (int l = 0; l < VN; ++l) f[k][l] = -INFINITY;
        }
      } else {
        const int e0 = j * VN - rv.a;
        if (j >= vlo && j < vhi) {
          // the window vector is in the stage; a vector straddling the row's start
          // or end keeps only the row's elements
          unpack<T>(*reinterpret_cast<const uint4*>(stage + j * 16), f[k]);
          if (e0 < 0 || e0 + VN > N) {
#pragma unroll
            for (int l = 0; l < VN; ++l)
              if (e0 + l < 0 || e0 + l >= N) f[k][l] = -INFINITY;
          }
        } else {
          // outside the copied span (the first or last vector of the whole matrix)
#pragma unroll
          for (int l = 0; l < VN; ++l) {
            const int e = e0 + l;
            f[k][l] = (j < rv.nv && e >= 0 && e < N) ? to_f(xr[e]) : -INFINITY;
          }
        }
      }
    }
    const RowStats st = block_row_stats<V, VN>(f, ok, post[it & 1]);
    if (!st.ok) return;  // the same decision in every warp
    // every thread has read its slice of the slot: refill it with a later row
    if (threadIdx.x == 0) {
      const int64_t nr = row + static_cast<int64_t>(stages) * gridDim.x;
      if (nr < M) issue(nr, slot);
    }
    const float scale = warp_scale(st.ml_warp, st.ml, st.d);

    T* yr = y + row * N;
    uint8_t* ywin = reinterpret_cast<uint8_t*>(reinterpret_cast<uintptr_t>(yr) - rv.a * sizeof(T));
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = threadIdx.x + k * blockDim.x;
      if (j >= rv.nv) continue;
      vscale<VN>(f[k], scale);
      const int e0 = j * VN - rv.a;
      if (kAligned || (y_vec && e0 >= 0 && e0 + VN <= N)) {
        st_stream(ywin + j * 16, pack<T>(f[k]));
      } else {
#pragma unroll
        for (int l = 0; l < VN; ++l)
          if (e0 + l >= 0 && e0 + l < N) yr[e0 + l] = from_f<T>(f[k][l]);
      }
    }
  }
}

// ------------------------------------------------------------------ variant 2: cluster

constexpr int kMaxCluster = 8;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t c;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(c));
  return c;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t c;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(c));
  return c;
}
// Every thread of every CTA of the cluster (used once, before the first remote store:
// every CTA is running and its barriers are initialised).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store v into CTA `peer`'s copy of *slot and count its 8 bytes on that CTA's copy of
// *bar (slot and bar sit at the same offsets in every CTA of the cluster).
__device__ __forceinline__ void dsmem_send(const float2* slot, const uint64_t* bar, uint32_t peer,
                                           float2 v) {
  uint32_t raddr, rbar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(smem_u32(slot)), "r"(peer));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(smem_u32(bar)), "r"(peer));
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];"
               :: "r"(raddr), "f"(v.x), "f"(v.y), "r"(rbar) : "memory");
}

// Row r of the matrix is processed by cluster (r mod clusters): CTA c of the cluster
// owns vectors [c*nvc, (c+1)*nvc) of the row's aligned window. Each CTA keeps its own
// ring of slice buffers, exactly as softmax_staged does for whole rows, and computes
// its slice's (max, sum) with one block barrier (block_row_stats). Thread 0 then sends
// that pair to every CTA of the cluster (st.async into slot [rank] of each CTA's
// array, completing 8 bytes on that CTA's mbarrier); each CTA waits (bounded) until
// all C pairs have landed and merges them in rank order, so every CTA normalises with
// the same bits: one exchange per row, and no cluster-wide barrier, so the row's
// streaming global stores never have to drain before it. Slots and mbarriers
// alternate between two sets by row parity: a CTA sends row r+2's pair only after it
// has received every CTA's pair of row r+1, which each CTA sends only after it has
// read its row-r slots. A CTA whose copy wait gave up sends a failure flag (a
// negative sum), and every CTA then leaves the loop at the same row; a CTA whose
// exchange wait gives up leaves too (its peers' waits then give up in turn).
template <typename T, int V, bool kAligned>
__global__ void __launch_bounds__(1024)
softmax_cluster(const T* __restrict__ x, T* __restrict__ y, int64_t M, int N, int nvc,
                int stages, uint32_t stage_bytes, unsigned* err) {
  constexpr int VN = Vec<T>::kN;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint8_t* ring = smem + 128;
  __shared__ float2 post[2][kWarp];
  __shared__ __align__(8) float2 c_stat[2][kMaxCluster];
  __shared__ __align__(8) uint64_t xbar[2];

  const int C = static_cast<int>(cluster_size());
  const int crank = static_cast<int>(cluster_rank());
  const int64_t first = cluster_id(), step = cluster_count();
  const uintptr_t xbase = reinterpret_cast<uintptr_t>(x);
  const uintptr_t xend = xbase + static_cast<uintptr_t>(M) * N * sizeof(T);
  const uintptr_t ok_lo = (xbase + 15) & ~uintptr_t(15);
  const uintptr_t ok_hi = xend & ~uintptr_t(15);
  const size_t row_bytes = static_cast<size_t>(N) * sizeof(T);
  const bool y_vec = ((reinterpret_cast<uintptr_t>(y) ^ xbase) & 15) == 0;
  const uint32_t xchg_bytes = static_cast<uint32_t>(C) * sizeof(float2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    for (int b = 0; b < 2; ++b) mbar_init(&xbar[b], 1);
    fence_mbar_init();
  }
  // every CTA of the cluster is running, with its barriers initialised, before any
  // CTA stores into another's shared memory
  cluster_sync_all();
  const uint64_t policy = l2_evict_first_policy();

  // this CTA's slice of a row window, clipped to the bytes a bulk copy may touch
  auto slice = [&](const RowView& rv, int& s0, int& s1, int& vlo, int& vhi) {
    s0 = crank * nvc;
    s1 = min(rv.nv, s0 + nvc);
    const uintptr_t cs0 = rv.win + static_cast<uintptr_t>(s0) * 16;
    const uintptr_t ce0 = rv.win + static_cast<uintptr_t>(s1) * 16;
    const uintptr_t cs = cs0 > ok_lo ? cs0 : ok_lo;
    const uintptr_t ce = ce0 < ok_hi ? ce0 : ok_hi;
    vlo = static_cast<int>((cs - rv.win) / 16);
    vhi = ce > cs ? static_cast<int>((ce - rv.win) / 16) : vlo;
  };
  auto issue = [&](int64_t row, int slot) {
    const RowView rv = row_view<T>(xbase + static_cast<uintptr_t>(row) * row_bytes, N);
    int s0, s1, vlo, vhi;
    slice(rv, s0, s1, vlo, vhi);
    if (vhi > vlo) {
      const uint32_t bytes = static_cast<uint32_t>(vhi - vlo) * 16;
      mbar_arrive_expect_tx(&full[slot], bytes);
      bulk_g2s(ring + size_t(slot) * stage_bytes + (vlo - s0) * 16,
               reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(vlo) * 16), bytes,
               &full[slot], policy);
    } else {
      mbar_arrive(&full[slot]);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      const int64_t r = first + static_cast<int64_t>(s) * step;
      if (r < M) issue(r, s);
    }
  }

  int it = 0;
  for (int64_t row = first; row < M; row += step, ++it) {
    const int slot = it % stages;
    const int par = it & 1;
    const uint32_t xphase = static_cast<uint32_t>((it >> 1) & 1);
    const bool ok = mbar_wait(&full[slot], static_cast<uint32_t>((it / stages) & 1), err);

    const RowView rv = row_view<T>(xbase + static_cast<uintptr_t>(row) * row_bytes, N);
    int s0, s1, vlo, vhi;
    slice(rv, s0, s1, vlo, vhi);
    if (kAligned) {
      vlo = s0;
      vhi = s1;
    }
    const uint8_t* stage = ring + size_t(slot) * stage_bytes;
    const T* xr = x + row * N;

    float f[V][VN];
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = s0 + static_cast<int>(threadIdx.x) + k * static_cast<int>(blockDim.x);
      const int e0 = j * VN - rv.a;
      if (j < s1 && j >= vlo && j < vhi) {
        unpack<T>(*reinterpret_cast<const uint4*>(stage + (j - s0) * 16), f[k]);
        if (!kAligned && (e0 < 0 || e0 + VN > N)) {
#pragma unroll
          for (int l = 0; l < VN; ++l)
            if (e0 + l < 0 || e0 + l >= N) f[k][l] = -INFINITY;
        }
      } else {
#pragma unroll
        for (int l = 0; l < VN; ++l) {
          const int e = e0 + l;
          f[k][l] = (j < s1 && e >= 0 && e < N) ? to_f(xr[e]) : -INFINITY;
        }
      }
    }
    // this CTA's (max, sum) of its slice, after one block barrier
    const RowStats st = block_row_stats<V, VN>(f, ok, post[par]);
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&xbar[par], xchg_bytes);
      for (int p = 0; p < C; ++p)
        dsmem_send(&c_stat[par][crank], &xbar[par], p, make_float2(st.ml, st.ok ? st.d : -1.f));
      const int64_t nr = row + static_cast<int64_t>(stages) * step;
      if (st.ok && nr < M) issue(nr, slot);
    }
    if (!mbar_wait(&xbar[par], xphase, err)) break;
    // merge the cluster's pairs in rank order: the same bits in every CTA
    float gml = -INFINITY;
    bool failed = false;
    for (int p = 0; p < C; ++p) {
      const float2 v = c_stat[par][p];
      gml = fmaxf(gml, v.x);
      failed |= v.y < 0.f;
    }
    if (failed) break;  // the same decision in every CTA of the cluster
    float gd = 0.f;
    for (int p = 0; p < C; ++p) {
      const float2 v = c_stat[par][p];
      if (v.x != -INFINITY) gd += v.y * ex2f(v.x - gml);
    }
    const float scale = warp_scale(st.ml_warp, gml, gd);

    T* yr = y + row * N;
    uint8_t* ywin = reinterpret_cast<uint8_t*>(reinterpret_cast<uintptr_t>(yr) - rv.a * sizeof(T));
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = s0 + static_cast<int>(threadIdx.x) + k * static_cast<int>(blockDim.x);
      if (j >= s1) continue;
      vscale<VN>(f[k], scale);
      const int e0 = j * VN - rv.a;
      if (kAligned || (y_vec && e0 >= 0 && e0 + VN <= N)) {
        st_stream(ywin + static_cast<size_t>(j) * 16, pack<T>(f[k]));
      } else {
#pragma unroll
        for (int l = 0; l < VN; ++l)
          if (e0 + l >= 0 && e0 + l < N) yr[e0 + l] = from_f<T>(f[k][l]);
      }
    }
  }
}

// ------------------------------------------------------------------ variant 2: two-pass

// Online-softmax state: ml = round(max * log2e), d = sum of exp2(x*log2e - ml).
// Every exponent is taken against a rounded ml with one FMA, and rescaling uses
// differences of the same rounded values, so all partial sums stay consistent with
// the final normalisation exp2(fma(x, log2e, -ml)).
__device__ __forceinline__ void online_merge(float& ml, float& d, float ml2, float d2) {
  const float mn = fmaxf(ml, ml2);
  if (mn == -INFINITY) return;
  d = d * ex2f(ml - mn) + d2 * ex2f(ml2 - mn);
  ml = mn;
}

template <typename T>
__global__ void __launch_bounds__(1024)
softmax_two_pass(const T* __restrict__ x, T* __restrict__ y, int N) {
  constexpr int VN = Vec<T>::kN;
  __shared__ float s_m[kWarp], s_d[kWarp];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * N;
  T* yr = y + row * N;
  const RowView rv = row_view<T>(reinterpret_cast<uintptr_t>(xr), N);
  const bool y_vec = ((reinterpret_cast<uintptr_t>(y) ^ reinterpret_cast<uintptr_t>(x)) & 15) == 0;

  // pass 1: online (max, sum); the row stays in L2 for pass 2 (normal priority)
  float m = -INFINITY, d = 0.f;  // m holds round(max * log2e)
  for (int j = threadIdx.x; j < rv.nv; j += blockDim.x) {
    const int e0 = j * VN - rv.a;
    float f[VN];
    if (e0 >= 0 && e0 + VN <= N) {
      unpack<T>(ld_keep(reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(j) * 16)), f);
    } else {
#pragma unroll
      for (int l = 0; l < VN; ++l)
        f[l] = (e0 + l >= 0 && e0 + l < N) ? to_f(xr[e0 + l]) : -INFINITY;
    }
    const float mn = fmaxf(m, vmax<VN>(f, -INFINITY) * kLog2e);
    const float2 s = vexp<VN>(f, make_float2(0.f, 0.f), -mn);
    d = (m == -INFINITY ? 0.f : d * ex2f(m - mn)) + (s.x + s.y);
    m = mn;
  }
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(kFull, m, o), d2 = __shfl_xor_sync(kFull, d, o);
    online_merge(m, d, m2, d2);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { s_m[wid] = m; s_d[wid] = d; }
  __syncthreads();
  const int nw = blockDim.x / kWarp;
  m = lane < nw ? s_m[lane] : -INFINITY;
  d = lane < nw ? s_d[lane] : 0.f;
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(kFull, m, o), d2 = __shfl_xor_sync(kFull, d, o);
    online_merge(m, d, m2, d2);
  }
  const float neg_ml = -m, inv = 1.f / d;

  // pass 2: normalise
  const uint64_t pol = evict_first_policy();
  uint8_t* ywin = reinterpret_cast<uint8_t*>(reinterpret_cast<uintptr_t>(yr) - rv.a * sizeof(T));
  for (int j = threadIdx.x; j < rv.nv; j += blockDim.x) {
    const int e0 = j * VN - rv.a;
    float f[VN];
    if (e0 >= 0 && e0 + VN <= N) {
      unpack<T>(ld_stream(reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(j) * 16), pol), f);
      vexp<VN>(f, make_float2(0.f, 0.f), neg_ml);
      vscale<VN>(f, inv);
      if (y_vec) {
        st_stream(ywin + static_cast<uintptr_t>(j) * 16, pack<T>(f));
        continue;
      }
    } else {
#pragma unroll
      for (int l = 0; l < VN; ++l)
        f[l] = (e0 + l >= 0 && e0 + l < N) ? ex2f(fmaf(to_f(xr[e0 + l]), kLog2e, neg_ml)) * inv : 0.f;
    }
#pragma unroll
    for (int l = 0; l < VN; ++l)
      if (e0 + l >= 0 && e0 + l < N) yr[e0 + l] = from_f<T>(f[l]);
  }
}

// ------------------------------------------------------------------ launch

struct StagedPlan {
  int threads, v, stages, ctas_per_sm;
  uint32_t stage_bytes;
};

// Every row starts on a 16-byte boundary and is a whole number of vectors.
template <typename T>
bool rows_aligned(const T* x, const T* y, int64_t N) {
  return reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
         (N * static_cast<int64_t>(sizeof(T))) % 16 == 0;
}

// Vectors per row window: N/VN when every row starts 16-byte aligned, else the
// worst case over row start offsets.
template <typename T>
int64_t window_vectors(bool aligned, int64_t N) {
  constexpr int VN = Vec<T>::kN;
  return aligned ? cdiv(N, VN) : (N + 2 * VN - 2) / VN;
}

// `max_ctas_per_sm` caps the CTAs the ring is sized for (the cluster kernel runs at
// 64 registers per thread, so at most 1024 threads per SM).
template <typename T>
StagedPlan plan_staged(int64_t nv_max, int max_ctas_per_sm = 32) {
  StagedPlan p{};
  // Cost of one row per CTA ~ threads * (V + 5): V vectors of element work plus a
  // fixed per-row share (two block reductions, the slot wait, the refill) worth about
  // five vectors. Fewer, fuller threads win for short rows.
  int64_t best = INT64_MAX;
  for (int t = 64; t <= 1024; t += 64) {
    const int64_t v = cdiv(nv_max, t);
    if (v > staged_max_v<T>()) continue;
    const int64_t cost = t * (v + 5);
    if (cost < best) {
      best = cost;
      p.threads = t;
      p.v = static_cast<int>(v);
    }
  }
  p.stage_bytes = static_cast<uint32_t>(cdiv(nv_max * 16, 128) * 128);
  // Most CTAs per SM (independent rows reducing at once) that still leaves each CTA
  // two ring slots, i.e. one row loading while one is reduced; a lone CTA may take
  // up to kMaxStages slots.
  const int64_t smem_per_sm = 220 * 1024;
  p.stages = 1;
  p.ctas_per_sm = 1;
  for (int c = std::min(2048 / p.threads, max_ctas_per_sm); c >= 1; --c) {
    const int64_t st = std::min<int64_t>(kMaxStages, smem_per_sm / c / (p.stage_bytes + 1024));
    if (st >= 2 || (c == 1 && st >= 1)) {
      p.stages = static_cast<int>(st);
      p.ctas_per_sm = c;
      break;
    }
  }
  return p;
}

template <typename T, int V, bool kAligned>
int launch_staged(const T* x, T* y, int64_t M, int64_t N, const StagedPlan& p, unsigned* err,
                  cudaStream_t s) {
  auto kern = softmax_staged<T, V, kAligned>;
  const size_t smem = 128 + size_t(p.stages) * p.stage_bytes;
  const void* fn = reinterpret_cast<const void*>(kern);
  if (int rc = ensure_dyn_smem(fn, static_cast<int>(smem))) return rc;
  int occ = 0;
  if (int rc = occupancy_blocks(fn, p.threads, smem, &occ)) return rc;
  if (occ < 1) return fail(KPB_ECUDA, "softmax: staged kernel does not fit on an SM");
  const int64_t grid = std::min<int64_t>(M, int64_t(sm_count()) * std::min(occ, p.ctas_per_sm));
  kern<<<static_cast<unsigned>(grid), p.threads, smem, s>>>(x, y, M, static_cast<int>(N),
                                                            p.stages, p.stage_bytes, err);
  KPB_LAUNCHED("softmax staged");
  return KPB_OK;
}

template <typename T, bool kAligned>
int dispatch_v(const T* x, T* y, int64_t M, int64_t N, const StagedPlan& p, unsigned* err,
               cudaStream_t s) {
  constexpr bool f32 = sizeof(T) == 4;
  switch (p.v) {
    case 1: return launch_staged<T, 1, kAligned>(x, y, M, N, p, err, s);
    case 2: return launch_staged<T, 2, kAligned>(x, y, M, N, p, err, s);
    case 3: return launch_staged<T, 3, kAligned>(x, y, M, N, p, err, s);
    case 4: return launch_staged<T, 4, kAligned>(x, y, M, N, p, err, s);
    case 5: return launch_staged<T, f32 ? 5 : 4, kAligned>(x, y, M, N, p, err, s);
    default: return launch_staged<T, f32 ? 6 : 4, kAligned>(x, y, M, N, p, err, s);
  }
}

template <typename T, int V, bool kAligned>
int launch_cluster(const T* x, T* y, int64_t M, int64_t N, int C, int nvc, const StagedPlan& p,
                   unsigned* err, cudaStream_t s) {
  auto kern = softmax_cluster<T, V, kAligned>;
  const size_t smem = 128 + size_t(p.stages) * p.stage_bytes;
  if (int rc = ensure_dyn_smem(reinterpret_cast<const void*>(kern), static_cast<int>(smem)))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(p.threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  // as many clusters as can be resident at once (at most one per row)
  cfg.gridDim = dim3(static_cast<unsigned>(C * sm_count()));
  int active = 0;
  if (int rc = occupancy_clusters(reinterpret_cast<const void*>(kern), cfg, C, &active)) return rc;
  if (active < 1) return fail(KPB_ECUDA, "softmax: cluster kernel does not fit");
  const int64_t clusters = std::min<int64_t>(M, active);
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * C));
  KPB_CUDA(cudaLaunchKernelEx(&cfg, kern, x, y, M, static_cast<int>(N), nvc, p.stages,
                              p.stage_bytes, err));
  return KPB_OK;
}

template <typename T, bool kAligned>
int dispatch_cluster(const T* x, T* y, int64_t M, int64_t N, int C, int nvc, const StagedPlan& p,
                     unsigned* err, cudaStream_t s) {
  constexpr bool f32 = sizeof(T) == 4;
  switch (p.v) {
    case 1: return launch_cluster<T, 1, kAligned>(x, y, M, N, C, nvc, p, err, s);
    case 2: return launch_cluster<T, 2, kAligned>(x, y, M, N, C, nvc, p, err, s);
    case 3: return launch_cluster<T, 3, kAligned>(x, y, M, N, C, nvc, p, err, s);
    case 4: return launch_cluster<T, 4, kAligned>(x, y, M, N, C, nvc, p, err, s);
    case 5: return launch_cluster<T, f32 ? 5 : 4, kAligned>(x, y, M, N, C, nvc, p, err, s);
    default: return launch_cluster<T, f32 ? 6 : 4, kAligned>(x, y, M, N, C, nvc, p, err, s);
  }
}

template <typename T>
int launch(int variant, const T* x, T* y, int64_t M, int64_t N, unsigned* err, cudaStream_t s) {
  if (M == 0 || N == 0) return KPB_OK;
  if (reinterpret_cast<uintptr_t>(x) % sizeof(T) || reinterpret_cast<uintptr_t>(y) % sizeof(T))
    return fail(KPB_EINVAL, "softmax: x and y must be element-aligned");
  if (variant == 0) {
    softmax_thread_row<T><<<static_cast<unsigned>(cdiv(M, 128)), 128, 0, s>>>(x, y, M, N);
    KPB_LAUNCHED("softmax variant 0");
    return KPB_OK;
  }
  if (variant == 1) {
    softmax_block_row<T><<<static_cast<unsigned>(M), 256, 0, s>>>(x, y, N);
    KPB_LAUNCHED("softmax variant 1");
    return KPB_OK;
  }
  const bool aligned = rows_aligned(x, y, N);
  const int64_t nv_max = window_vectors<T>(aligned, N);
  const int64_t cta_max = 1024 * staged_max_v<T>();  // vectors one CTA keeps in registers
  if (nv_max > cta_max) {
    // The smallest cluster that holds the row at up to 1024 threads a CTA. Measured on
    // bf16 [4096, 131072]: clusters of 4 x 1024 threads 4.38 TB/s, 8 x 512 4.06,
    // 16 x 256 (four CTAs per SM) 3.73: every CTA of a cluster waits each row for the
    // slowest one, and that costs more as clusters grow than extra CTAs per SM hide.
    int C = 2;
    while (C < kMaxCluster && cdiv(nv_max, C) > cta_max) C *= 2;
    if (cdiv(nv_max, C) <= cta_max) {
      const int nvc = static_cast<int>(cdiv(nv_max, C));
      StagedPlan p = plan_staged<T>(nvc);
      p = plan_staged<T>(nvc, std::max(1, 1024 / p.threads));
      return aligned ? dispatch_cluster<T, true>(x, y, M, N, C, nvc, p, err, s)
                     : dispatch_cluster<T, false>(x, y, M, N, C, nvc, p, err, s);
    }
    softmax_two_pass<T><<<static_cast<unsigned>(M), 1024, 0, s>>>(x, y, static_cast<int>(N));
    KPB_LAUNCHED("softmax two-pass");
    return KPB_OK;
  }
  const StagedPlan p = plan_staged<T>(nv_max);
  return aligned ? dispatch_v<T, true>(x, y, M, N, p, err, s)
                 : dispatch_v<T, false>(x, y, M, N, p, err, s);
}

}  // namespace

int softmax(int variant, int dtype, const void* x, void* y, int64_t M, int64_t N,
            unsigned* err, cudaStream_t s) {
  switch (dtype) {
    case KPB_F32:
      return launch(variant, static_cast<const float*>(x), static_cast<float*>(y), M, N, err, s);
    case KPB_F16:
      return launch(variant, static_cast<const __half*>(x), static_cast<__half*>(y), M, N, err, s);
    case KPB_BF16:
      return launch(variant, static_cast<const __nv_bfloat16*>(x),
                    static_cast<__nv_bfloat16*>(y), M, N, err, s);
    default: return fail(KPB_EINVAL, "softmax: unknown dtype " + std::to_string(dtype));
  }
}

}  // namespace kpb
