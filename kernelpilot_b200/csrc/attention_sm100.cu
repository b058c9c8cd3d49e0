// tcgen05 flash-attention forward for kp.attention / kp.attention_causal variant 1
// (fp16/bf16, head dim 64 or 128): O = softmax(Q K^T / sqrt(D)) V per (batch, head),
// fp32 softmax statistics, fp32 accumulation in tensor memory.
//
// Replaces kernelpilot's csrc/kernels/attention.hip attn_flash (:62-110: one thread
// per query, K/V tiles of 32 in shared memory, scalar FMAs, D=128 spills) with:
//   * one CTA per (head, 128-query tile); causal tiles run heaviest first;
//   * warp 0 (one lane): TMA loads of Q once and of K_j / V_j (128 keys x D, 128-byte
//     swizzle, 3-D tensor maps so rows past S read as zeros) into two 2-slot rings;
//   * warp 1 (one lane): tcgen05.mma issue, in the order S_0, S_1, PV_0, S_2, PV_1 ...
//     S_j = Q K_j^T lands in one of two 128-column fp32 TMEM buffers, so the tensor
//     core computes S_{j+1} while the softmax works on S_j; O += P_j V_j accumulates in
//     TMEM (D columns);
//   * warps 2-5: one thread per query row. Reads its S row from TMEM twice (max, then
//     exp2/sum) in 32-column chunks, keeps the running max in log2 units and only
//     rescales O (TMEM load/scale/store of its row) when the max grows by more than
//     2^8, writes P as bf16/fp16 into a 128-byte-swizzled K-major tile that is the A
//     operand of the PV MMA; at the end O / l -> global.
// Masking: keys >= S, and keys > query on the causal diagonal tile, score -inf.
#include <cudaTypedefs.h>

#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {

namespace {

constexpr int BQ = 128, BKV = 128;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 softmax
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.f;  // log2 units: rescale O when max grows by > 256x

template <int D>
struct AttnSmem {
  static constexpr int kTile = BQ * D * 2;         // Q, K_j or V_j tile (BQ == BKV)
  static constexpr int kP = BQ * BKV * 2;          // P tile
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;            // 2 slots
  static constexpr int kV = kK + 2 * kTile;        // 2 slots
  static constexpr int kPOff = kV + 2 * kTile;
  static constexpr int kPLoOff = kPOff + kP;       // rounding residual of P (few-key tiles)
  static constexpr int kRed = kPLoOff + kP;       // row max / sum exchange, 4 x 128 floats
  static constexpr int kBar = kRed + 4 * 128 * 4;
  static constexpr int kBytes = kBar + 256;        // + barriers (base is 1024-aligned)
};

// 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled tile of 128-byte rows.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

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

// Barrier over the 64 threads of a warp pair that also ANDs a predicate across them,
// so both warps take every exit decision together.
__device__ __forceinline__ bool pair_all(int id, bool p) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred pi, po;\n\t"
               "setp.ne.u32 pi, %1, 0;\n\t"
               "bar.red.and.pred po, %2, 64, pi;\n\t"
               "selp.u32 %0, 1, 0, po;\n\t}"
               : "=r"(r) : "r"(static_cast<uint32_t>(p)), "r"(id) : "memory");
  return r != 0;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
               :: "r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <typename T, int D, bool kCausal>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
            const __grid_constant__ CUtensorMap tv, T* __restrict__ o, int S, float scale_log2,
            unsigned* err) {
  using L = AttnSmem<D>;
  constexpr int kAtoms = D / 64;              // 64-wide (128-byte) column atoms per row
  constexpr int kAtomBytes = BQ * 128;        // one atom column of a 128-row tile
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) uint8_t smem[];
  // the 128-byte swizzle atoms need a 1024-byte aligned base; the layout leaves no
  // room to realign, so report a misaligned base instead of computing garbage
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicOr(err, kErrSmemAlign);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint64_t* drain = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_qt = static_cast<int>(gridDim.x);
  const int qt = kCausal ? n_qt - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y;
  const int q0 = qt * BQ;
  const int nkv_all = (S + BKV - 1) / BKV;
  const int nkv = kCausal ? min(nkv_all, qt + 1) : nkv_all;
  // Rows that see only a handful of keys (the first causal tile, or very short
  // sequences) carry P as bf16/fp16 hi + lo parts: two PV MMAs instead of one, so the
  // rounding of P does not dominate their error.
  const bool split = (kCausal && qt == 0) || S <= 256;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 11; ++i) mbar_init(&bars[i], 1);
    mbar_init(p_full, 256);
    mbar_init(pv_done, 1);
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
  const uint32_t tmem_o = tmem + 2 * BKV;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA loads
      mbar_arrive_expect_tx(q_full, L::kTile);
#pragma unroll
      for (int a = 0; a < kAtoms; ++a)
        tma_load_3d(smem + L::kQ + a * kAtomBytes, &tq, a * 64, q0, bh, q_full);
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int slot = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[slot], ph, err)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[slot], L::kTile);
#pragma unroll
        for (int a = 0; a < kAtoms; ++a)
          tma_load_3d(smem + L::kK + slot * L::kTile + a * kAtomBytes, &tk, a * 64, j * BKV, bh,
                      &k_full[slot]);
        if (!mbar_wait(&v_empty[slot], ph, err)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[slot], L::kTile);
#pragma unroll
        for (int a = 0; a < kAtoms; ++a)
          tma_load_3d(smem + L::kV + slot * L::kTile + a * kAtomBytes, &tv, a * 64, j * BKV, bh,
                      &v_full[slot]);
      }
      // drain: every issued copy has been consumed
      if (ok) {
        for (int j = max(0, nkv - 2); j < nkv; ++j) {
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&k_empty[j & 1], ph, err)) break;
          if (!mbar_wait(&v_empty[j & 1], ph, err)) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issue
      constexpr uint32_t idesc_s = idesc_f16(BQ, BKV, kBf16, false, false);
      constexpr uint32_t idesc_o = idesc_f16(BQ, D, kBf16, false, true);
      const uint32_t q_addr = smem_u32(smem + L::kQ);
      const uint32_t p_addr = smem_u32(smem + L::kPOff);
      const uint32_t plo_addr = smem_u32(smem + L::kPLoOff);
      bool ok = mbar_wait(q_full, 0, err);
      auto issue_s = [&](int j) -> bool {
        const int slot = j & 1;
        if (!mbar_wait(&k_full[slot], (j >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kK + slot * L::kTile);
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t off = (s / 4) * kAtomBytes + (s % 4) * 32;
          umma_f16_ss(tmem + slot * BKV, smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + off, 16, 1024), idesc_s, s > 0 ? 1u : 0u);
        }
        umma_commit(&k_empty[slot]);
        umma_commit(&s_full[slot]);
        return true;
      };
      if (ok && nkv > 0) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(p_full, j & 1, err)) { ok = false; break; }
        const int slot = j & 1;
        if (!mbar_wait(&v_full[slot], (j >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + L::kV + slot * L::kTile);
#pragma unroll
        for (int s = 0; s < BKV / 16; ++s) {
          const uint64_t pd = smem_desc_sw128(p_addr + (s / 4) * kAtomBytes + (s % 4) * 32, 16, 1024);
          const uint64_t vd = smem_desc_sw128(v_addr + s * 16 * 128, kAtomBytes, 1024);
          umma_f16_ss(tmem_o, pd, vd, idesc_o, (j > 0 || s > 0) ? 1u : 0u);
        }
        if (split) {
#pragma unroll
          for (int s = 0; s < BKV / 16; ++s) {
            const uint64_t pd = smem_desc_sw128(plo_addr + (s / 4) * kAtomBytes + (s % 4) * 32, 16, 1024);
            const uint64_t vd = smem_desc_sw128(v_addr + s * 16 * 128, kAtomBytes, 1024);
            umma_f16_ss(tmem_o, pd, vd, idesc_o, 1u);
          }
        }
        umma_commit(&v_empty[slot]);
        umma_commit(pv_done);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ------------------------------------------------ softmax + epilogue (warps 2..9)
    // Two warps per TMEM lane quarter: warp w owns rows 32*(w%4) .. +31 and key
    // columns [64*half, 64*half + 64) of each S tile, half = (w - 2) / 4. The pair
    // shares the row max through shared memory behind a 64-thread named barrier.
    const int quarter = warp % 4;
    const int half = (warp - 2) / 4;
    const int t = quarter * 32 + lane;          // query row within the tile (= TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t col_s = half * (BKV / 2);    // this warp's S / P columns
    const uint32_t col_o = half * (D / 2);      // this warp's O columns
    const int pair_bar = 1 + quarter;
    const int q = q0 + t;
    const uint32_t p_hi = smem_u32(smem + L::kPOff) + half * kAtomBytes;
    const uint32_t p_lo = smem_u32(smem + L::kPLoOff) + half * kAtomBytes;
    float* red = reinterpret_cast<float*>(smem + L::kRed);  // [2 parities][2 halves][128 rows]
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int slot = j & 1;
      const bool s_ready = mbar_wait(&s_full[slot], (j >> 1) & 1, err);
      tc_fence_after();
      const int k0 = j * BKV;
      uint32_t r[2][32];
      tmem_ld32(tmem + lane_base + slot * BKV + col_s, r[0]);
      tmem_ld32(tmem + lane_base + slot * BKV + col_s + 32, r[1]);
      tmem_wait_ld();
      // masking only on tiles that reach past S or cross the causal diagonal
      const bool edge = (k0 + BKV > S) || (kCausal && j == qt);
      if (edge) {
        int kend = min(S, k0 + BKV);
        if (kCausal) kend = min(kend, q + 1);
        const int nvalid = kend - k0 - static_cast<int>(col_s);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i >= nvalid) r[c][i] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        mx0 = max3f(mx0, __uint_as_float(r[0][i]), __uint_as_float(r[0][i + 1]));
        mx1 = max3f(mx1, __uint_as_float(r[1][i]), __uint_as_float(r[1][i + 1]));
      }
      float mx = fmaxf(mx0, mx1);
      red[(slot * 2 + half) * BQ + t] = mx;
      ok = pair_all(pair_bar, s_ready);
      if (!ok) break;
      mx = fmaxf(mx, red[(slot * 2 + (half ^ 1)) * BQ + t]);
      const float mrow = mx * scale_log2;
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
      float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float2 a = __ffma2_rn(make_float2(__uint_as_float(r[c][i]), __uint_as_float(r[c][i + 1])),
                                sc2, mn2);
          if ((i & 7) == 6) {
            a = exp2_poly2(a);  // one pair in four on the FMA pipe: relieves the MUFU
          } else {
            a.x = ex2_approx(a.x);
            a.y = ex2_approx(a.y);
          }
          r[c][i] = __float_as_uint(a.x);
          r[c][i + 1] = __float_as_uint(a.y);
          if (i & 2) ls1 = __fadd2_rn(ls1, a); else ls0 = __fadd2_rn(ls0, a);
        }
      l += (ls0.x + ls0.y) + (ls1.x + ls1.y);
      // P buffers and O are free once PV_{j-1} completed
      if (j > 0) {
        ok = pair_all(pair_bar, mbar_wait(pv_done, (j - 1) & 1, err));
        if (!ok) break;
        tc_fence_after();
      }
      if (__any_sync(kFull, rescale_o)) {
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t o_r[32];
          tmem_ld32(tmem_o + lane_base + col_o + c * 32, o_r);
          tmem_wait_ld();
          const float f = rescale_o ? corr : 1.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) o_r[i] = __float_as_uint(__uint_as_float(o_r[i]) * f);
          tmem_st32(tmem_o + lane_base + col_o + c * 32, o_r);
        }
        tmem_wait_st();
      }
      // this warp's 64 keys fill one 128-byte swizzle atom of the P tile: 8 chunks
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const int chunk = c * 4 + h;
          uint32_t w[4], wl[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a = __uint_as_float(r[c][8 * h + 2 * e]);
            const float b = __uint_as_float(r[c][8 * h + 2 * e + 1]);
            w[e] = pack2<T>(a, b);
            if (split) {
              const float2 hv = unpack2<T>(w[e]);
              wl[e] = pack2<T>(a - hv.x, b - hv.y);
            }
          }
          st_shared_v4(p_hi + sw128(t, chunk), w[0], w[1], w[2], w[3]);
          if (split) st_shared_v4(p_lo + sw128(t, chunk), wl[0], wl[1], wl[2], wl[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // epilogue: O / l -> global; the row sum is the pair's two partial sums
    if (ok && nkv > 0) {
      red[((nkv & 1) * 2 + half) * BQ + t] = l;  // the parity buffer block nkv-1 did not use
      ok = pair_all(pair_bar, mbar_wait(pv_done, (nkv - 1) & 1, err));
      l += red[((nkv & 1) * 2 + (half ^ 1)) * BQ + t];
    }
    if (ok && nkv > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = o + (static_cast<int64_t>(bh) * S + q) * D + col_o;
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) {
        uint32_t rr[32];
        tmem_ld32(tmem_o + lane_base + col_o + c * 32, rr);
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
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// (BH, S, D) 16-bit tensor as a 3-D TMA map with (64 x 128 x 1) boxes, 128-byte swizzle.
int make_tmap_bhsd(CUtensorMap* map, const void* base, bool bf16, int64_t BH, int64_t S,
                   int64_t D);

namespace {

template <typename T, int D, bool kCausal>
int launch_attn(const T* q, const T* k, const T* v, T* o, int64_t BH, int64_t S,
                unsigned* err, cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv;
  if (int rc = make_tmap_bhsd(&mq, q, bf16, BH, S, D)) return rc;
  if (int rc = make_tmap_bhsd(&mk, k, bf16, BH, S, D)) return rc;
  if (int rc = make_tmap_bhsd(&mv, v, bf16, BH, S, D)) return rc;
  auto kern = attn_fwd_tc<T, D, kCausal>;
  const int smem = AttnSmem<D>::kBytes;
  KPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const dim3 grid(static_cast<unsigned>(cdiv(S, BQ)), static_cast<unsigned>(BH));
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  kern<<<grid, kThreads, smem, s>>>(mq, mk, mv, o, static_cast<int>(S), scale_log2, err);
  KPB_LAUNCHED("attention tcgen05");
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
