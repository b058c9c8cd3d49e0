// tcgen05 GEMM for kp.matmul variant 3 with fp16/bf16 inputs: C = A @ B, row-major
// A (M, K), B (K, N), C (M, N), fp32 accumulation in tensor memory.
//
// Replaces the SIMT "vectorized" stage of kernelpilot's csrc/kernels/matmul.hip
// (mm_vec :142-208, CUDA-core FFMA) with a Blackwell design:
//   * persistent grid, one CTA per SM, tiles of 128 x 256 visited in bands of
//     kGroupM M-blocks so the A and B panels in flight stay resident in L2;
//   * warp 0 (one lane) streams 128x64 A tiles and 64x256 B tiles with TMA into a
//     kStages-deep shared-memory ring (128-byte swizzle; A is K-major, B is N-major);
//   * warp 1 (one lane) issues tcgen05.mma (M=128, N=256, K=16) into one of two
//     256-column fp32 accumulators in TMEM and releases ring slots / accumulators
//     with tcgen05.commit;
//   * warps 2-9 drain the other accumulator (tcgen05.ld -> bf16/fp16 -> global)
//     while the next tile accumulates; two warps share each 32-lane TMEM quarter
//     and take alternate 32-column chunks.
// Every mbarrier wait is bounded; a timeout sets the error word and the roles shut
// down in order (wait for issued copies and MMAs, free TMEM, exit).
//
// Shapes TMA cannot describe (a row pitch that is not a multiple of 16 bytes, e.g.
// N = 4097, or an unaligned base) are first copied into a zero-padded, aligned
// workspace; C is written with masked stores, so any M, N, K works.
#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 4;
constexpr int kABytes = BM * BK * 2;        // 16 KB
constexpr int kBBoxBytes = BK * 64 * 2;     // one 64(K) x 64(N) box, 8 KB
constexpr int kBBytes = BK * BN * 2;        // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr int kGroupM = 16;
constexpr uint32_t kTmemCols = 512;         // two 128 x 256 fp32 accumulators
constexpr int kEpiBytes = kEpiWarps * 32 * 17 * 4;  // epilogue transpose staging
constexpr int kSmemBytes = kStages * kStageBytes + 256 + kEpiBytes + 1024;  // + barriers + alignment

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int group = kGroupM * num_n;
  const int first_m = (t / group) * kGroupM;
  const int rows = min(num_m - first_m, kGroupM);
  const int r = t % group;
  mb = first_m + r % rows;
  nb = r / rows;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2_t(float a, float b) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const uint32_t (&r)[32], int valid,
                                            bool vec_ok) {
  float f[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]);
  if (vec_ok && valid >= 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = pack<T>(f + 8 * i);
      *reinterpret_cast<uint4*>(dst + 8 * i) = v;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = from_f<T>(f[i]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
        T* __restrict__ C, int M, int N, int K, int64_t ldc, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint32_t* stage_out = reinterpret_cast<uint32_t*>(smem + kStages * kStageBytes + 256);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps * 32);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      pdl_wait_primary();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err)) { ok = false; break; }
          uint8_t* sa = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sa, &tmA, kb * BK, mb * BM, &full[stage]);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(sa + kABytes + j * kBBoxBytes, &tmB, nb * BN + j * 64, kb * BK,
                        &full[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      // every slot released once more = every copy issued has landed and been consumed
      for (int s = 0; s < kStages && ok; ++s) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err)) break;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16(BM, BN, std::is_same<T, __nv_bfloat16>::value,
                                           false, true);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, err)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * kStageBytes);
          const uint32_t b0 = a0 + kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + k * 16 * 128, kBBoxBytes, 1024);
            umma_f16_ss(d, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 and the
    // 32-column chunks c = (w-2)/4, +2, +4, ...
    const int quarter = warp % 4;
    const int chunk0 = (warp - 2) / 4;
    const int r_in_tile = quarter * 32 + lane;
    const bool vec_ok = (ldc % 8 == 0) && (reinterpret_cast<uintptr_t>(C) % 16 == 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const bool ok = mbar_wait(&tfull[acc], acc_phase, err);
      if (!__all_sync(kFull, ok)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(mb) * BM + r_in_tile;
      T* crow = C + row * ldc;
#pragma unroll 1
      for (int c = chunk0; c < BN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + c * 32, r);
        tmem_wait_ld();
        const int col0 = nb * BN + c * 32;
        if (vec_ok) {
          if (row < M && col0 < N) store_row32<T>(crow + col0, r, N - col0, true);
        } else if (col0 < N) {
          // C rows are not 16-byte aligned: transpose the warp's 32x32 chunk through
          // shared memory so each store instruction writes 32 consecutive elements of
          // one row (row stride 17 words: conflict-free in both directions)
          uint32_t* st = stage_out + (warp - 2) * (32 * 17);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            st[lane * 17 + i] = pack2_t<T>(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          __syncwarp();
          const int64_t row0 = static_cast<int64_t>(mb) * BM + quarter * 32;
          const bool col_ok = col0 + lane < N;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const uint32_t w = st[rr * 17 + lane / 2];
            const uint16_t h = static_cast<uint16_t>((lane & 1) ? (w >> 16) : (w & 0xFFFF));
            if (col_ok && row0 + rr < M)
              *reinterpret_cast<uint16_t*>(C + (row0 + rr) * ldc + col0 + lane) = h;
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ CTA-pair kernel
//
// The same roles on a cluster of two CTAs on two SMs (cta_group::2). A pair computes a
// 256 x 256 tile: CTA r loads rows [128 r, 128 r + 128) of the A block and columns
// [128 r, 128 r + 128) of the B block into its own shared memory (plain TMA, one
// tile per CTA, nothing broadcast), and the leader CTA's MMA thread issues
// M = 256, N = 256 MMAs that read A and B from both CTAs and accumulate each CTA's
// 128 rows in that CTA's TMEM. Against one CTA with 128 x 256 tiles, each SM stages
// half as much of B per output (32 KB stages instead of 48 KB, so six stages fit) and
// the L2 serves half the B traffic.
//   * both CTAs' copies of stage s complete on the LEADER's full[s] (the peer's TMA
//     names the leader's barrier); the leader's producer expects both CTAs' bytes;
//   * the MMA commits arrive on empty[s] and tfull[acc] in BOTH CTAs (commit with a
//     two-CTA mask), so each producer and each epilogue waits on its own barriers;
//   * every epilogue warp of both CTAs arrives on the leader's tempty[acc] once it
//     has drained its columns (16 arrivals), which the MMA thread waits for;
//   * TMEM is allocated and freed by warp 1 of both CTAs together, after a cluster
//     barrier at the end, when no MMA reads the peer's shared memory any more.
constexpr int kPairStages = 6;
constexpr int kPairBM = 256, kPairBN = 256;
constexpr int kPairBHalf = 128;                           // B columns per CTA
constexpr int kPairABytes = 128 * BK * 2;                 // 16 KB
constexpr int kPairBBytes = BK * kPairBHalf * 2;          // 16 KB (two 64 x 64 boxes)
constexpr int kPairStageBytes = kPairABytes + kPairBBytes;
constexpr int kPairEpiArrivals = 2 * kEpiWarps;           // one per epilogue warp, both CTAs
constexpr int kPairSmemBytes = kPairStages * kPairStageBytes + 256 + kEpiBytes + 1024;
static_assert(kPairSmemBytes <= 227 * 1024, "pair GEMM shared memory");

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             T* __restrict__ C, int M, int N, int K, int64_t ldc, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint32_t* stage_out = reinterpret_cast<uint32_t*>(smem + kPairStages * kPairStageBytes + 256);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cta_rank_in_cluster();
  const bool leader = rank == 0;
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  const int num_m = (M + kPairBM - 1) / kPairBM, num_n = (N + kPairBN - 1) / kPairBN;
  const int tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kPairEpiArrivals);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
    tc_fence_before();
  }
  // both CTAs' barriers are initialised (and TMEM allocated) before either CTA's
  // copies or commits can reach the other
  cluster_barrier();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs): this CTA's half of A and of B
      // (after a pitch copy this grid starts early as its programmatic dependent: the
      // set-up above overlaps the copy's tail, the first load waits for its result)
      pdl_wait_primary();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err)) { ok = false; break; }
          uint8_t* sa = smem + stage * kPairStageBytes;
          const uint32_t bar = cluster_map(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kPairStageBytes);
          tma_load_2d_pair(sa, &tmA, kb * BK, mb * kPairBM + static_cast<int>(rank) * 128, bar);
#pragma unroll
          for (int j = 0; j < kPairBHalf / 64; ++j)
            tma_load_2d_pair(sa + kPairABytes + j * kBBoxBytes, &tmB,
                             nb * kPairBN + static_cast<int>(rank) * kPairBHalf + j * 64, kb * BK,
                             bar);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
      }
      // every slot released once more = every copy issued has landed and been consumed
      for (int s = 0; s < kPairStages && ok; ++s) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err)) break;
        if (++stage == kPairStages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA only)
      constexpr uint32_t idesc = idesc_f16(kPairBM, kPairBN, std::is_same<T, __nv_bfloat16>::value,
                                           false, true);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, err)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * kPairBN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * kPairStageBytes);
          const uint32_t b0 = a0 + kPairABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + k * 16 * 128, kBBoxBytes, 1024);
            umma_f16_ss_pair(d, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
        umma_commit_pair(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of the pair's tile
    const int quarter = warp % 4;
    const int chunk0 = (warp - 2) / 4;
    const int r_in_tile = static_cast<int>(rank) * 128 + quarter * 32 + lane;
    const bool vec_ok = (ldc % 8 == 0) && (reinterpret_cast<uintptr_t>(C) % 16 == 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < tiles; t += npairs) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const bool ok = mbar_wait(&tfull[acc], acc_phase, err);
      if (!__all_sync(kFull, ok)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(mb) * kPairBM + r_in_tile;
      T* crow = C + row * ldc;
#pragma unroll 1
      for (int c = chunk0; c < kPairBN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kPairBN + c * 32, r);
        tmem_wait_ld();
        const int col0 = nb * kPairBN + c * 32;
        if (vec_ok) {
          if (row < M && col0 < N) store_row32<T>(crow + col0, r, N - col0, true);
        } else if (col0 < N) {
          uint32_t* st = stage_out + (warp - 2) * (32 * 17);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            st[lane * 17 + i] = pack2_t<T>(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          __syncwarp();
          const int64_t row0 = static_cast<int64_t>(mb) * kPairBM + rank * 128 + quarter * 32;
          const bool col_ok = col0 + lane < N;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const uint32_t w = st[rr * 17 + lane / 2];
            const uint16_t h = static_cast<uint16_t>((lane & 1) ? (w >> 16) : (w & 0xFFFF));
            if (col_ok && row0 + rr < M)
              *reinterpret_cast<uint16_t*>(C + (row0 + rr) * ldc + col0 + lane) = h;
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_map(&tempty[acc], 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  __syncthreads();
  // no CTA leaves (or frees TMEM) while the pair's MMAs may still touch its memory
  cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// dst (rows x cols_pad) = src (rows x cols) with zero columns appended; cols_pad is a
// multiple of 8, so every thread writes aligned 16-byte vectors of a dst row.
// Interior vectors read the two aligned 16-byte words that cover them and shift the
// row's 2-byte misalignment out with funnel shifts; vectors at row or buffer ends
// fall back to masked 2-byte loads. A CTA of kPadThreads takes whole rows (rows
// blockIdx.x, + gridDim.x, ...), and each thread issues the loads of kPadUnroll
// vectors before it stores any, so a row's loads are in flight together.
constexpr int kPadThreads = 128;
constexpr int kPadUnroll = 4;

__device__ __forceinline__ uint32_t word_at(const uint4& a, const uint4& b, int i) {
  switch (i) {
    case 0: return a.x; case 1: return a.y; case 2: return a.z; case 3: return a.w;
    case 4: return b.x; case 5: return b.y; case 6: return b.z; default: return b.w;
  }
}

template <typename T>
__global__ void __launch_bounds__(kPadThreads)
pad_cols(const T* __restrict__ src, T* __restrict__ dst, int64_t rows, int64_t cols,
         int64_t cols_pad) {
  // the GEMM that reads dst may launch now; its loads wait for this grid to finish
  pdl_launch_dependents();
  const int64_t nvec = cols_pad / 8;
  const uintptr_t src_lo = reinterpret_cast<uintptr_t>(src);
  const uintptr_t src_hi = src_lo + static_cast<uintptr_t>(rows * cols) * 2;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* s = src + r * cols;
    uint4* d = reinterpret_cast<uint4*>(dst + r * cols_pad);
    const uintptr_t rs = reinterpret_cast<uintptr_t>(s);
    const uintptr_t base = rs & ~uintptr_t(15);
    const int off = static_cast<int>(rs - base);  // even, 0..14
    const int q = off >> 2, sh = (off & 3) * 8;
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += kPadUnroll * kPadThreads) {
      uint4 lo[kPadUnroll], hi[kPadUnroll];
      bool fast[kPadUnroll];
#pragma unroll
      for (int k = 0; k < kPadUnroll; ++k) {
        const int64_t v = v0 + k * kPadThreads;
        const uintptr_t w0 = base + static_cast<uintptr_t>(v) * 16;
        fast[k] = v < nvec && v * 8 + 8 <= cols && w0 >= src_lo && w0 + 32 <= src_hi;
        if (fast[k]) {
          lo[k] = *reinterpret_cast<const uint4*>(w0);
          hi[k] = *reinterpret_cast<const uint4*>(w0 + 16);
        }
      }
#pragma unroll
      for (int k = 0; k < kPadUnroll; ++k) {
        const int64_t v = v0 + k * kPadThreads;
        if (v >= nvec) continue;
        if (fast[k]) {
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = __funnelshift_r(word_at(lo[k], hi[k], q + i), word_at(lo[k], hi[k], q + i + 1), sh);
          d[v] = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
          uint16_t e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t c = v * 8 + i;
            e[i] = c < cols ? reinterpret_cast<const uint16_t*>(s)[c] : uint16_t(0);
          }
          d[v] = make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                            e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
        }
      }
    }
  }
}

}  // namespace

int make_tmap_2d_sw128(CUtensorMap* map, const void* base, bool bf16, uint64_t inner,
                       uint64_t outer, uint64_t pitch_bytes, uint32_t box_outer);

namespace {

struct Staging {
  bool pad_a, pad_b;
  int64_t kp, np;
  size_t a_bytes, b_bytes;
};

Staging staging(const void* A, const void* B, int64_t M, int64_t N, int64_t K) {
  Staging s{};
  s.pad_a = (K % 8 != 0) || (reinterpret_cast<uintptr_t>(A) % 16 != 0);
  s.pad_b = (N % 8 != 0) || (reinterpret_cast<uintptr_t>(B) % 16 != 0);
  // staged pitches are whole 128-byte lines, so every 128-byte TMA box row is one line
  s.kp = cdiv(K, 64) * 64;
  s.np = cdiv(N, 64) * 64;
  s.a_bytes = s.pad_a ? static_cast<size_t>(cdiv(M * s.kp * 2, 256) * 256) : 0;
  s.b_bytes = s.pad_b ? static_cast<size_t>(cdiv(K * s.np * 2, 256) * 256) : 0;
  return s;
}

template <typename T>
int launch_tc(const T* A, const T* B, T* C, int64_t M, int64_t N, int64_t K, void* ws,
              size_t ws_bytes, unsigned* err, cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const Staging st = staging(A, B, M, N, K);
  if (st.a_bytes + st.b_bytes > 0 &&
      (ws == nullptr || ws_bytes < st.a_bytes + st.b_bytes ||
       reinterpret_cast<uintptr_t>(ws) % 16 != 0))
    return fail(KPB_EINVAL, "matmul: workspace missing or too small for the aligned staging copy");
  const T* a = A;
  const T* b = B;
  int64_t lda = K, ldb = N;
  uint8_t* w = static_cast<uint8_t*>(ws);
  const int sms = sm_count();
  if (st.pad_a) {
    T* ap = reinterpret_cast<T*>(w);
    pad_cols<T><<<static_cast<unsigned>(std::min<int64_t>(M, 1 << 16)), kPadThreads, 0, s>>>(A, ap, M, K, st.kp);
    KPB_LAUNCHED("matmul pad A");
    a = ap;
    lda = st.kp;
    w += st.a_bytes;
  }
  if (st.pad_b) {
    T* bp = reinterpret_cast<T*>(w);
    pad_cols<T><<<static_cast<unsigned>(std::min<int64_t>(K, 1 << 16)), kPadThreads, 0, s>>>(B, bp, K, N, st.np);
    KPB_LAUNCHED("matmul pad B");
    b = bp;
    ldb = st.np;
  }
  CUtensorMap ta, tb, tb_pair;
  if (int rc = make_tmap_2d_sw128(&ta, a, bf16, static_cast<uint64_t>(lda), M, lda * 2, BM)) return rc;
  if (int rc = make_tmap_2d_sw128(&tb, b, bf16, static_cast<uint64_t>(ldb), K, ldb * 2, BK)) return rc;
  tb_pair = tb;  // the same 64 x 64 boxes of B
  // with a padded A the K loop runs over the zero-padded width (B reads zeros there)
  if (M > BM) {
    auto kern = gemm_tc_pair<T>;
    if (int rc = ensure_dyn_smem(reinterpret_cast<const void*>(kern), kPairSmemBytes)) return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (st.pad_a || st.pad_b) ? 2 : 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kPairSmemBytes;
    cfg.stream = s;
    cfg.gridDim = dim3(static_cast<unsigned>(sms / 2 * 2));
    int active = 0;
    if (int rc = occupancy_clusters(reinterpret_cast<const void*>(kern), cfg, 2, &active)) return rc;
    if (active < 1) return fail(KPB_ECUDA, "matmul: the CTA-pair kernel does not fit");
    const int64_t pair_tiles = cdiv(M, kPairBM) * cdiv(N, kPairBN);
    const int64_t pairs = std::min<int64_t>(pair_tiles, active);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    KPB_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb_pair, C, static_cast<int>(M),
                                static_cast<int>(N), static_cast<int>(lda), N, err));
    return KPB_OK;
  }
  auto kern = gemm_tc<T>;
  if (int rc = ensure_dyn_smem(reinterpret_cast<const void*>(kern), kSmemBytes)) return rc;
  const int64_t tiles = cdiv(M, BM) * cdiv(N, BN);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (st.pad_a || st.pad_b) ? 1 : 0;
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(tiles, sms)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  KPB_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, C, static_cast<int>(M), static_cast<int>(N),
                              static_cast<int>(lda), N, err));
  return KPB_OK;
}

}  // namespace

size_t matmul_tc_workspace_bytes(int dtype, int64_t M, int64_t N, int64_t K) {
  if (dtype == KPB_F32) return 0;
  // worst case (unaligned base pointers as well): both staging copies
  const Staging s = staging(reinterpret_cast<const void*>(1), reinterpret_cast<const void*>(1),
                            M, N, K);
  return s.a_bytes + s.b_bytes;
}

int matmul_tc(int dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
              void* ws, size_t ws_bytes, unsigned* err, cudaStream_t s) {
  if (dtype == KPB_BF16)
    return launch_tc(static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B),
                     static_cast<__nv_bfloat16*>(C), M, N, K, ws, ws_bytes, err, s);
  if (dtype == KPB_F16)
    return launch_tc(static_cast<const __half*>(A), static_cast<const __half*>(B),
                     static_cast<__half*>(C), M, N, K, ws, ws_bytes, err, s);
  return KPB_EUNSUPPORTED;
}

}  // namespace kpb
