// tcgen05 flash-attention forward for kp.attention / kp.attention_causal variant 1
// (fp16/bf16, head dim 64 or 128): O = softmax(Q K^T / sqrt(D)) V per (batch, head),
// fp32 softmax statistics, fp32 accumulation in tensor memory.
//
// Replaces kernelpilot's csrc/kernels/attention.hip attn_flash (:62-110: one thread
// per query, K/V tiles of 32 in shared memory, scalar FMAs, D=128 spills) with a
// two-tile ping-pong design:
//   * one CTA per (head, 256 queries) = two 128-query tiles A and B that share every
//     K/V tile; causal CTAs run heaviest first;
//   * warp 0 (one lane): TMA loads of Q_A, Q_B once and of K_j / V_j (128 keys x D,
//     128-byte swizzle; 3-D tensor maps, so rows past S read as zeros) into a 2-slot
//     ring, K_j and V_j of a block under one barrier;
//   * warp 1 (one lane): tcgen05.mma issue in the order
//       S_A0 S_B0 | PV_A0 S_A1 PV_B0 S_B1 | PV_A1 S_A2 PV_B1 S_B2 | ...
//     S_t = Q_t K_j^T lands in TMEM (128 fp32 columns per tile); P_t is written back
//     over the first 64 columns of S_t as packed bf16/fp16 pairs and PV_t = P_t V_j
//     reads it straight from TMEM (the A-from-TMEM form of tcgen05.mma), accumulating
//     O_t in TMEM. While one tile's softmax runs, the tensor core works on the other;
//   * warps 4-11 (tile A) and 12-19 (tile B): two threads per query row, one per key
//     half (64 of the block's 128 scores each, read from TMEM in one go); they swap
//     their half-row maxima through shared memory (one 64-thread named barrier per
//     block); running max in log2 units; O is rescaled (TMEM load/scale/store, half
//     the columns each) only when the max grows by more than 2^8;
//     five eighths of the exponentials run on the MUFU (ex2.approx) and three eighths
//     on the FMA pipe (exp2_poly2); P is packed and stored 32 keys at a time, and the
//     row sum is taken after P has been handed to the tensor core (it is not on the
//     S -> P -> PV -> S chain); at the end O / l -> global.
// A tcgen05.commit tracks every MMA issued before it, so "S_t(j) is ready" also means
// PV_t(j-1) has finished: the softmax never waits on the PV separately.
// Masking: keys >= S, and keys > query on the causal diagonal tile, score -inf.
// Rows that see only a handful of keys (the first causal CTA, or S <= 256) carry P
// as hi + lo parts (P - rounded P in columns 64..127 of S_t) and take a second PV MMA,
// so the rounding of P does not dominate their error.
#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {

namespace {

constexpr int BQ = 128, BKV = 128;
constexpr int kTiles = 2;                   // query tiles per CTA
// warpgroup 0: TMA, MMA, 2 idle; warpgroups 1-2: tile A; 3-4: tile B. Each query row
// is shared by two warps of its tile (keys 0..63 and 64..127 of every block), which
// exchange only the block's row max.
constexpr int kThreads = 640;
// Register split (setmaxnreg): the launch gives 640 x 96; warpgroup 0 drops to 56 and
// the four softmax warpgroups rise to 104: 128*56 + 512*104 = 60416 <= 640*96 = 61440,
// and each scheduler holds one producer and four softmax warps: (56 + 4*104) * 32 <= 16384.
constexpr uint32_t kRegsProducer = 56, kRegsSoftmax = 104;
constexpr uint32_t kTmemCols = 512;         // S_A | S_B | O_A | O_B, 128 columns each
constexpr float kRescaleThreshold = 8.f;    // log2 units: rescale O when max grows > 256x

template <int D>
struct AttnSmem {
  static constexpr int kTile = BQ * D * 2;  // a Q tile, or a K_j / V_j tile (BQ == BKV)
  static constexpr int kQ = 0;              // kTiles tiles
  static constexpr int kK = kQ + kTiles * kTile;  // 2 slots
  static constexpr int kV = kK + 2 * kTile;       // 2 slots
  static constexpr int kBar = kV + 2 * kTile;
  // row-max exchange between the two warps of a row: [block parity][tile][half][row]
  // floats, then the same layout of ok flags, then the half-row sums for the epilogue
  static constexpr int kX = kBar + 256;
  static constexpr int kXMax = 0, kXOk = 2 * kTiles * 2 * BQ * 4, kXSum = 2 * kXOk;
  static constexpr int kBytes = kX + kXSum + kTiles * 2 * BQ * 4;  // base is 1024-byte aligned
};

// 2^x on the multi-function unit (ex2.approx.ftz: max relative error ~2^-22).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for two lanes on the FMA pipe: x = n + f with n = round(x) (added to 1.5*2^23 so
// the rounded integer lands in the low mantissa bits), f in [-1/2, 1/2],
// 2^f ~ c0 + f (c1 + f (c2 + f c3)) (coefficients from fit_exp2_poly.py: minimax
// relative error 7.5e-5, far below the bf16/fp16 rounding P gets next), then n is
// added to the exponent field. Inputs are <= 8 here; below -126 they clamp to
// -126, so masked (-inf) scores give ~1e-38 rather than 0, which no output can see.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = __fadd2_rn(x, make_float2(kMagic, kMagic));
  const float2 n = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 p = __ffma2_rn(make_float2(0.0551716685295105f, 0.0551716685295105f), f,
                        make_float2(0.2426111251115799f, 0.2426111251115799f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  const int nx = __float_as_int(t.x) - 0x4B400000, ny = __float_as_int(t.y) - 0x4B400000;
  return make_float2(__int_as_float(__float_as_int(p.x) + (nx << 23)),
                     __int_as_float(__float_as_int(p.y) + (ny << 23)));
}

// Two values as one 32-bit TMEM column of the A operand (first value in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (std::is_same<T, __half>::value)
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  else
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// kSplit: the CTAs whose rows see only a handful of keys carry P as hi + lo (a separate
// instantiation, launched on its own small grid: the extra live registers of the lo
// part would otherwise spill in every CTA). A CTA's 256-query block is
// ct_first + ct_step * blockIdx.x.
template <typename T, int D, bool kCausal, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
            const __grid_constant__ CUtensorMap tv, T* __restrict__ o, int S, float scale_log2,
            int ct_first, int ct_step, unsigned* err) {
  using L = AttnSmem<D>;
  constexpr int kAtoms = D / 64;              // 64-wide (128-byte) column atoms per row
  constexpr int kAtomBytes = BQ * 128;        // one atom column of a 128-row tile
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) uint8_t smem[];
  // the 128-byte swizzle atoms need a 1024-byte aligned base; the layout leaves no
  // room to realign, so report a misaligned base instead of computing garbage
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicOr(err, kErrSmemAlign);
    if (kSplit) pdl_wait_primary();
    return;
  }
  // the few-key grid that follows a causal main grid may start on SMs this grid no
  // longer needs (its rows are disjoint; it waits for this grid before it completes)
  if (!kSplit) pdl_launch_dependents();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  // K_j and V_j travel together: one barrier per ring slot for both (every wait of
  // the MMA-issuing thread costs the tensor core a bubble, so it waits once per block)
  uint64_t* kv_full = bars + 1;  // [2]
  uint64_t* kv_empty = bars + 3; // [2]
  uint64_t* s_full = bars + 5;   // [tile]
  uint64_t* p_full = bars + 7;   // [tile]
  uint64_t* pv_done = bars + 9;  // [tile]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ct = ct_first + ct_step * static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y;
  const int q0 = ct * kTiles * BQ;
  const int nkv_all = (S + BKV - 1) / BKV;
  // KV blocks each tile needs (0 for a tile that lies wholly past S)
  auto tile_nkv = [&](int t) {
    const int qt = ct * kTiles + t;
    return q0 + t * BQ >= S ? 0 : (kCausal ? min(nkv_all, qt + 1) : nkv_all);
  };
  const int nkv0 = tile_nkv(0), nkv1 = tile_nkv(1);
  auto nkv = [&](int t) { return t == 0 ? nkv0 : nkv1; };
  const int nkv_max = max(nkv0, nkv1);
  constexpr bool split = kSplit;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);  // q_full, kv_full, kv_empty, s_full
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&p_full[t], 256);  // every softmax thread of the tile
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRegsProducer));
    if (warp == 0) {
      if (lane == 0) {
        // ------------------------------------------------ TMA loads
        mbar_arrive_expect_tx(q_full, kTiles * L::kTile);
#pragma unroll
        for (int t = 0; t < kTiles; ++t)
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            tma_load_3d(smem + L::kQ + t * L::kTile + a * kAtomBytes, &tq, a * 64, q0 + t * BQ, bh,
                        q_full);
        bool ok = true;
        for (int j = 0; j < nkv_max && ok; ++j) {
          const int slot = j & 1;
          const uint32_t ph = ((j >> 1) & 1) ^ 1;
          if (!mbar_wait(&kv_empty[slot], ph, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[slot], 2 * L::kTile);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            tma_load_3d(smem + L::kK + slot * L::kTile + a * kAtomBytes, &tk, a * 64, j * BKV, bh,
                        &kv_full[slot]);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            tma_load_3d(smem + L::kV + slot * L::kTile + a * kAtomBytes, &tv, a * 64, j * BKV, bh,
                        &kv_full[slot]);
        }
        // drain: every issued copy has been consumed
        if (ok) {
          for (int j = max(0, nkv_max - 2); j < nkv_max; ++j) {
            const uint32_t ph = (j >> 1) & 1;
            if (!mbar_wait(&kv_empty[j & 1], ph, err)) break;
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // ------------------------------------------------ MMA issue
        constexpr uint32_t idesc_s = idesc_f16(BQ, BKV, kBf16, false, false);
        constexpr uint32_t idesc_o = idesc_f16(BQ, D, kBf16, false, true);
        const uint32_t q_addr = smem_u32(smem + L::kQ);
        // K_j / V_j are last read by the MMAs of the last tile that still needs block j;
        // the slot is released after that tile's PV (its S was issued before)
        auto k_last = [&](int t, int j) { return t == kTiles - 1 || j >= nkv1; };
        auto issue_s = [&](int t, int j) {
          const int slot = j & 1;
          const uint32_t k_addr = smem_u32(smem + L::kK + slot * L::kTile);
          const uint32_t qa = q_addr + t * L::kTile;
#pragma unroll
          for (int s = 0; s < D / 16; ++s) {
            const uint32_t off = (s / 4) * kAtomBytes + (s % 4) * 32;
            umma_f16_ss(tmem + t * BKV, smem_desc_sw128(qa + off, 16, 1024),
                        smem_desc_sw128(k_addr + off, 16, 1024), idesc_s, s > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[t]);
        };
        auto issue_pv = [&](int t, int j) {
          const int slot = j & 1;
          const uint32_t v_addr = smem_u32(smem + L::kV + slot * L::kTile);
          const uint32_t p_tmem = tmem + t * BKV;           // P_t: 64 packed columns
          const uint32_t o_tmem = tmem + (kTiles + t) * BKV;
#pragma unroll
          for (int s = 0; s < BKV / 16; ++s)
            umma_f16_ts(o_tmem, p_tmem + s * 8, smem_desc_sw128(v_addr + s * 16 * 128, kAtomBytes, 1024),
                        idesc_o, (j > 0 || s > 0) ? 1u : 0u);
          if (split) {
#pragma unroll
            for (int s = 0; s < BKV / 16; ++s)
              umma_f16_ts(o_tmem, p_tmem + 64 + s * 8,
                          smem_desc_sw128(v_addr + s * 16 * 128, kAtomBytes, 1024), idesc_o, 1u);
          }
          umma_commit(&pv_done[t]);
          if (k_last(t, j)) umma_commit(&kv_empty[slot]);
        };
        bool ok = mbar_wait(q_full, 0, err);
        if (ok && nkv_max > 0) {
          ok = mbar_wait(&kv_full[0], 0, err);
          tc_fence_after();
          if (ok) {
            for (int t = 0; t < kTiles; ++t)
              if (nkv(t) > 0) issue_s(t, 0);
          }
        }
        for (int j = 0; j < nkv_max && ok; ++j) {
          // K_j / V_j were waited for before S(j) was issued
          bool k_next_ready = false;
          for (int t = 0; t < kTiles && ok; ++t) {
            if (j >= nkv(t)) continue;
            if (!mbar_wait(&p_full[t], j & 1, err)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, j);
            if (j + 1 < nkv(t)) {
              if (!k_next_ready) {
                if (!mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, err)) { ok = false; break; }
                tc_fence_after();
                k_next_ready = true;
              }
              issue_s(t, j + 1);
            }
          }
        }
        umma_commit(drain);
        mbar_wait(drain, 0, err);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(kRegsSoftmax));
    // ------------------------------------------------ softmax + epilogue
    const int sw = warp - 4;                    // softmax warp 0..15
    const int tile = sw / 8;
    const int half = (sw / 4) & 1;              // keys 64*half .. 64*half+63 of every block
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;        // query row within the tile (= TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem + lane_base + tile * BKV;
    const uint32_t o_tmem = tmem + lane_base + (kTiles + tile) * BKV + half * (D / 2);
    const int qt = ct * kTiles + tile;
    const int q = q0 + tile * BQ + row;
    const int my_nkv = nkv(tile);
    // exchange slots: this thread's and its partner's (same row, other key half)
    float* xmax = reinterpret_cast<float*>(smem + L::kX + L::kXMax);
    int* xok = reinterpret_cast<int*>(smem + L::kX + L::kXOk);
    float* xsum = reinterpret_cast<float*>(smem + L::kX + L::kXSum);
    const int x_me = (tile * 2 + half) * BQ + row, x_peer = (tile * 2 + 1 - half) * BQ + row;
    constexpr int kXStride = kTiles * 2 * BQ;   // one block parity
    // named barrier of the row's two warps; both always reach it together (the ok flags
    // travel through the exchange, so a failed wait ends the loop in both warps at once)
    const int bar_id = 1 + tile * 4 + quarter;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < my_nkv; ++j) {
      const bool got = __all_sync(kFull, mbar_wait(&s_full[tile], j & 1, err));
      const int k0 = j * BKV + half * 64;
      uint32_t r[2][32];
      float hmax = -INFINITY;
      if (got) {
        tc_fence_after();
        tmem_ld32(s_tmem + half * 64, r[0]);
        tmem_ld32(s_tmem + half * 64 + 32, r[1]);
        tmem_wait_ld();
        // masking only on blocks that reach past S or cross the causal diagonal
        const bool edge = (j * BKV + BKV > S) || (kCausal && j == qt);
        if (edge) {
          int kend = S;
          if (kCausal) kend = min(kend, q + 1);
          const int nvalid = kend - k0;
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i >= nvalid) r[c][i] = __float_as_uint(-INFINITY);
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            mx[2 * c] = max3f(mx[2 * c], __uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1]));
            mx[2 * c + 1] = max3f(mx[2 * c + 1], __uint_as_float(r[c][i + 2]), __uint_as_float(r[c][i + 3]));
          }
        hmax = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3]));
      }
      const int xb = (j & 1) * kXStride;
      xmax[xb + x_me] = hmax;
      xok[xb + x_me] = got ? 1 : 0;
      asm volatile("bar.sync %0, 64;" :: "r"(bar_id) : "memory");
      const float pmax = xmax[xb + x_peer];
      ok = got && xok[xb + x_peer] != 0;
      if (!ok) break;
      const float mrow = fmaxf(hmax, pmax) * scale_log2;
      float corr = 1.f;
      bool rescale_o = false;
      if (mrow > m_used + kRescaleThreshold || (m_used == -INFINITY && mrow > -INFINITY)) {
        corr = (m_used == -INFINITY) ? 0.f : ex2_approx(m_used - mrow);
        rescale_o = j > 0 && m_used != -INFINITY;
        l *= corr;
        m_used = mrow;
      }
      const float mneg = (m_used == -INFINITY) ? 0.f : -m_used;
      const float2 sc2 = make_float2(scale_log2, scale_log2), mn2 = make_float2(mneg, mneg);
      // exponentials, 32 keys at a time, each chunk packed into P as soon as it is done
      // (this half's 64 keys: packed columns 32*half.. of S); for few-key rows also
      // P - rounded P (columns 64 + 32*half..). The row sum waits until P has been
      // handed to the tensor core.
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float2 a = __ffma2_rn(make_float2(__uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1])),
                                sc2, mn2);
          const int pair = (i / 2) & 7;
          if (pair == 1 || pair == 4 || pair == 6) {
            a = exp2_poly2(a);  // three pairs in eight on the FMA pipe: relieves the MUFU
          } else {
            a.x = ex2_approx(a.x);
            a.y = ex2_approx(a.y);
          }
          r[c][i] = __float_as_uint(a.x);
          r[c][i + 1] = __float_as_uint(a.y);
        }
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          w[e] = pack2<T>(__uint_as_float(r[c][2 * e]), __uint_as_float(r[c][2 * e + 1]));
        tmem_st16(s_tmem + half * 32 + c * 16, w);
        if (split) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float2 hv = unpack2<T>(w[e]);
            w[e] = pack2<T>(__uint_as_float(r[c][2 * e]) - hv.x,
                            __uint_as_float(r[c][2 * e + 1]) - hv.y);
          }
          tmem_st16(s_tmem + 64 + half * 32 + c * 16, w);
        }
      }
      // PV_t(j-1) is complete (covered by the commit behind s_full), so O can be
      // rescaled; each of the row's two threads scales half of O's columns
      if (__any_sync(kFull, rescale_o)) {
        // 16 columns at a time: the block's 64 P values stay live for the row sum
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o_r[16];
          tmem_ld16(o_tmem + c * 16, o_r);
          tmem_wait_ld();
          const float f = rescale_o ? corr : 1.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) o_r[i] = __float_as_uint(__uint_as_float(o_r[i]) * f);
          tmem_st16(o_tmem + c * 16, o_r);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[tile]);
      // this half's share of the row sum, while the tensor core runs PV_t(j) and S_t(j+1)
      float2 ls[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        ls[c] = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          ls[c] = __fadd2_rn(ls[c], make_float2(__uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1])));
      }
      l += (ls[0].x + ls[0].y) + (ls[1].x + ls[1].y);
    }
    // epilogue: both halves' sums -> O / l -> global, each thread half of the row
    if (my_nkv > 0) {
      const bool done =
          ok && __all_sync(kFull, mbar_wait(&pv_done[tile], (my_nkv - 1) & 1, err));
      xsum[x_me] = done ? l : -1.f;  // a sum is never negative: -1 = this half failed
      asm volatile("bar.sync %0, 64;" :: "r"(bar_id) : "memory");
      const float l_peer = xsum[x_peer];
      if (done && l_peer >= 0.f) {
        tc_fence_after();
        const float lsum = l + l_peer;
        const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
        T* orow = o + (static_cast<int64_t>(bh) * S + q) * D + half * (D / 2);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + c * 32, rr);
          tmem_wait_ld();
          if (q < S) {
            float f[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(rr[i]) * inv;
#pragma unroll
            for (int h = 0; h < 4; ++h)
              *reinterpret_cast<uint4*>(orow + c * 32 + 8 * h) = pack<T>(f + 8 * h);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // launched as a programmatic dependent of the main grid: complete only after it, so
  // work queued behind this grid on the stream sees the whole output
  if (kSplit) pdl_wait_primary();
}

}  // namespace

// (BH, S, D) 16-bit tensor as a 3-D TMA map with (64 x 128 x 1) boxes, 128-byte swizzle.
int make_tmap_bhsd(CUtensorMap* map, const void* base, bool bf16, int64_t BH, int64_t S,
                   int64_t D, uint32_t box_rows);

namespace {

template <typename T, int D, bool kCausal>
int launch_attn(const T* q, const T* k, const T* v, T* o, int64_t BH, int64_t S,
                unsigned* err, cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv;
  if (int rc = make_tmap_bhsd(&mq, q, bf16, BH, S, D, 128)) return rc;
  if (int rc = make_tmap_bhsd(&mk, k, bf16, BH, S, D, 128)) return rc;
  if (int rc = make_tmap_bhsd(&mv, v, bf16, BH, S, D, 128)) return rc;
  const int smem = AttnSmem<D>::kBytes;
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  const int n_ct = static_cast<int>(cdiv(S, kTiles * BQ));
  // few-key rows: every block when S <= 256, else the first causal block of each head
  const int n_split = S <= kTiles * BQ ? n_ct : (kCausal ? 1 : 0);
  if (n_ct > n_split) {
    // causal: heaviest blocks first
    auto kern = attn_fwd_tc<T, D, kCausal, false>;
    if (int rc = ensure_dyn_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
    const dim3 grid(static_cast<unsigned>(n_ct - n_split), static_cast<unsigned>(BH));
    kern<<<grid, kThreads, smem, s>>>(mq, mk, mv, o, static_cast<int>(S), scale_log2,
                                      kCausal ? n_ct - 1 : n_split, kCausal ? -1 : 1, err);
    KPB_LAUNCHED("attention tcgen05");
  }
  if (n_split > 0) {
    auto kern = attn_fwd_tc<T, D, kCausal, true>;
    if (int rc = ensure_dyn_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(n_split), static_cast<unsigned>(BH));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    // after a main grid: programmatic dependent launch, so these CTAs fill the SMs
    // the main grid's last CTAs leave idle (without a main grid, griddepcontrol.wait
    // returns at once)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = n_ct > n_split ? 1 : 0;
    KPB_CUDA(cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, o, static_cast<int>(S), scale_log2, 0, 1,
                                err));
    KPB_LAUNCHED("attention tcgen05 few-key rows");
  }
  return KPB_OK;
}

template <typename T, bool kCausal>
int attn_tc_d(const void* q, const void* k, const void* v, void* o, int64_t BH, int64_t S,
              int64_t D, unsigned* err, cudaStream_t s) {
  auto qq = static_cast<const T*>(q), kk = static_cast<const T*>(k), vv = static_cast<const T*>(v);
  auto oo = static_cast<T*>(o);
  if (D == 64) return launch_attn<T, 64, kCausal>(qq, kk, vv, oo, BH, S, err, s);
  if (D == 128) return launch_attn<T, 128, kCausal>(qq, kk, vv, oo, BH, S, err, s);
  return KPB_EUNSUPPORTED;
}

}  // namespace

int attention_tc(int dtype, bool causal, const void* q, const void* k, const void* v, void* o,
                 int64_t BH, int64_t S, int64_t D, unsigned* err, cudaStream_t s) {
  if (D != 64 && D != 128) return KPB_EUNSUPPORTED;
  if (S >= (int64_t{1} << 31) / BQ) return KPB_EUNSUPPORTED;
  const uintptr_t bases = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                          reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o);
  if (bases % 16 != 0) return KPB_EUNSUPPORTED;  // TMA and vector stores need 16-byte bases
  if (dtype == KPB_BF16)
    return causal ? attn_tc_d<__nv_bfloat16, true>(q, k, v, o, BH, S, D, err, s)
                  : attn_tc_d<__nv_bfloat16, false>(q, k, v, o, BH, S, D, err, s);
  if (dtype == KPB_F16)
    return causal ? attn_tc_d<__half, true>(q, k, v, o, BH, S, D, err, s)
                  : attn_tc_d<__half, false>(q, k, v, o, BH, S, D, err, s);
  return KPB_EUNSUPPORTED;
}

}  // namespace kpb
