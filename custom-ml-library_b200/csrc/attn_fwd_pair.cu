// Prefill attention forward on tcgen05 with TWO 128-row query tiles per CTA
// (bf16 / f16, D = Dv in {64, 128}).  Same arithmetic as tc_fwd_kernel
// (tensorsmith nn/attention.py:175-198: running max, running sum, rescaled
// accumulator, output a / l, LSE = m + log l), scheduled so that the tensor
// pipe has one query tile's MMAs to run while the other tile's softmax runs.
//
// One CTA = query tiles t = 0, 1 (rows q0 .. q0+255) of one (batch, head).
// Both tiles read the same K/V tiles, so every K/V tile comes from L2 once
// per 256 query rows.  Warp roles:
//   warp 0   TMA producer: Q0, Q1 once; then K(j), V(j) alternately into one
//            ring of tile-sized slots (K and V tiles share the slots)
//   warp 1   MMA issuer (one thread), order per key tile j:
//              P0(j).V(j) -> O0,  S0(j+1) = Q0 K(j+1)^T,
//              P1(j).V(j) -> O1,  S1(j+1) = Q1 K(j+1)^T
//            S_t and P_t share TMEM columns; P_t (bf16/f16 pairs) is the A
//            operand of P.V, read from tensor memory
//   warp 2   TMEM allocator: S0 | S1 | O0 | O1 (512 columns)
//   warps 4-7   softmax of query tile 0, warps 8-11 of query tile 1: thread r
//            owns row r (TMEM lane r) and the full 128-key row of each tile.
// Because S_t(j+1) is issued after P_t(j).V(j), the completion of S_t(j+1)
// implies that O_t holds every earlier product: the softmax thread rescales
// O_t in TMEM (lazily, when its running max grew by more than 2^8) between
// reading S_t(j+1) and releasing P_t(j+1), with no further barrier.  The two
// softmax warpgroups run half a period apart, each one's exponentials
// overlapping the other tile's MMAs.  Warpgroup 0 (producer, MMA issuer,
// allocator) runs on 56 registers a thread so that the softmax warpgroups
// hold a 128-key row of scores, its 64 packed probabilities and the running
// state in 216 without spilling.  No TMA load uses cluster multicast.
#include <type_traits>

#include "ptx.cuh"
#include "tc_fwd.cuh"
#include "tc_util.cuh"

namespace tsa {

namespace {

constexpr int kBM = 128, kBN = 128;
constexpr int kSlabBytes = 128 * 128;  // 128 rows x 128 bytes
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr uint32_t kFaultSmemAlign = 0x108;
constexpr int kMaxStages = 10;

template <int D> struct PairCfg {
  static constexpr int kSlabs = D / 64;
  static constexpr int kTileBytes = kSlabs * kSlabBytes;  // one 128-row Q/K/V tile
  static constexpr int kStages = D == 128 ? 5 : 10;       // K/V ring slots
  static constexpr int kOffQ = 0;                          // Q0, Q1
  static constexpr int kOffKV = 2 * kTileBytes;
  static constexpr int kOffBar = kOffKV + kStages * kTileBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kSlack = 1024;  // alignment of the tile base to 1024 bytes
  static constexpr int kSmem = kOffBar + kBarBytes + kSlack;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColS = 0;    // S0, S1: 128 columns each
  static constexpr uint32_t kColO = 256;  // O0, O1: D columns each
  static_assert(kSmem <= 232448, "shared memory");
  static_assert(kStages <= kMaxStages, "barriers");
};

struct PairBars {
  uint64_t q_full[2];
  uint64_t kv_full[kMaxStages], kv_empty[kMaxStages];
  uint64_t s_full[2];  // S_t(j) landed in TMEM (one phase per key tile)
  uint64_t p_full[2];  // softmax of tile t wrote P_t(j) (4 warp arrivals)
  uint64_t o_done[2];  // the last P_t.V of tile t completed
  uint64_t drain;
  uint32_t tmem_base;
};
static_assert(sizeof(PairBars) <= 256, "barrier block");

struct PairArgs {
  ts_attn_params p;
  int n_units;  // ceil(q_len / 256) per (batch, head)
  uint32_t* fault;
  DropoutArgs drop;  // kDrop instantiation only
};

// Key tiles visible to query rows [r0, r0 + 128) (0 when the tile is empty).
__device__ __forceinline__ int visible_tiles(const ts_attn_params& p, int r0, int kv_end, int64_t offset) {
  if (r0 >= p.q_len) return 0;
  int lim = kv_end;
  if (p.is_causal) {
    const int r_last = min(r0 + kBM - 1, p.q_len - 1);
    lim = (int)i64max(0, i64min(kv_end, (int64_t)r_last + offset + 1));
  }
  return ceil_div(lim, kBN);
}

}  // namespace

template <int D, bool kBF16, bool kDrop>
__global__ void __launch_bounds__(384, 1)
    tc_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, PairArgs args) {
  using C = PairCfg<D>;
  constexpr int S = C::kStages;
  const ts_attn_params& p = args.p;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t pad = (1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad > (uint32_t)C::kSlack) {  // uniform for the CTA: nothing initialised yet
    if (threadIdx.x == 0) record_fault(args.fault, kFaultSmemAlign);
    return;
  }
  unsigned char* smem = smem_raw + pad;
  PairBars* bars = reinterpret_cast<PairBars*>(smem + C::kOffBar);
  unsigned char* sQ = smem + C::kOffQ;
  unsigned char* sKV = smem + C::kOffKV;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = args.n_units - 1 - (int)blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.q_heads / p.kv_heads);
  const int q0 = unit * 2 * kBM;

  int kv_end = p.kv_len;
  int64_t offset = p.causal_offset;
  if (p.kv_lens) {
    kv_end = min(kv_end, max(0, p.kv_lens[b]));
    offset = (int64_t)kv_end - p.q_len;
  }
  const int n_t[2] = {visible_tiles(p, q0, kv_end, offset), visible_tiles(p, q0 + kBM, kv_end, offset)};
  const int n_max = max(n_t[0], n_t[1]);
  const bool dead = fault_set(args.fault);

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      ptx::mbar_init(&bars->q_full[t], 1);
      ptx::mbar_init(&bars->s_full[t], 1);
      ptx::mbar_init(&bars->p_full[t], 4);
      ptx::mbar_init(&bars->o_done[t], 1);
    }
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&bars->kv_full[s], 1);
      ptx::mbar_init(&bars->kv_empty[s], 1);
    }
    ptx::mbar_init(&bars->drain, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 2) {
    ptx::tmem_alloc(&bars->tmem_base, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Fill f of the K/V ring: K(f/2) for even f, V(f/2) for odd f; slot f % S.
  auto slot_addr = [&](int f) -> unsigned char* { return sKV + (f % S) * C::kTileBytes; };

  if (warp < 4) {
    // Registers: 384 threads x 168 at launch; this warpgroup gives back to
    // 56 and the softmax warpgroups grow to 216 (4 x 32 x 56 + 8 x 32 x 216 =
    // 62464 <= 64512).  One setmaxnreg site per warpgroup role.
    ptx::setmaxnreg_dec<56>();
    if (warp == 0) {
      // ---------------------------- producer ------------------------------
      if (lane == 0 && n_max > 0 && !dead) {
        ptx::prefetch_tensormap(&tm_q);
        ptx::prefetch_tensormap(&tm_k);
        ptx::prefetch_tensormap(&tm_v);
        for (int t = 0; t < 2; ++t) {
          if (n_t[t] == 0) continue;
          ptx::mbar_expect_tx(&bars->q_full[t], C::kTileBytes);
          for (int s = 0; s < C::kSlabs; ++s)
            ptx::tma_load_4d(sQ + t * C::kTileBytes + s * kSlabBytes, &tm_q, 64 * s, q0 + t * kBM, h, b,
                             &bars->q_full[t]);
        }
        int issued = 0;
        for (int f = 0; f < 2 * n_max; ++f) {
          const int s = f % S;
          if (f >= S && !wait_bar(&bars->kv_empty[s], ((f / S) - 1) & 1, args.fault, FAULT_FWD_EMPTY)) break;
          ptx::mbar_expect_tx(&bars->kv_full[s], C::kTileBytes);
          const CUtensorMap* map = (f & 1) ? &tm_v : &tm_k;
          for (int sl = 0; sl < C::kSlabs; ++sl)
            ptx::tma_load_4d(slot_addr(f) + sl * kSlabBytes, map, 64 * sl, (f >> 1) * kBN, hk, b,
                             &bars->kv_full[s]);
          issued = f + 1;
        }
        // Drain: every issued copy must have landed before shared memory is released.
        for (int t = 0; t < 2; ++t)
          if (n_t[t] > 0) (void)wait_bar(&bars->q_full[t], 0, nullptr, FAULT_FWD_DRAIN);
        for (int f = max(0, issued - S); f < issued; ++f)
          (void)wait_bar(&bars->kv_full[f % S], (f / S) & 1, nullptr, FAULT_FWD_DRAIN);
      }
    } else if (warp == 1) {
      // ---------------------------- MMA issuer ----------------------------
      if (lane == 0 && n_max > 0 && !dead) {
        constexpr uint32_t idesc_qk = ptx::idesc_f16(kBF16, kBM, kBN, false, false);
        constexpr uint32_t idesc_pv = ptx::idesc_f16(kBF16, kBM, D, false, true);
        const uint32_t sQa = ptx::smem_u32(sQ);
        bool ok = true;
        for (int t = 0; t < 2 && ok; ++t)
          if (n_t[t] > 0) ok = wait_bar(&bars->q_full[t], 0, args.fault, FAULT_FWD_Q);
        // S_t(j) = Q_t K(j)^T into S_t.
        auto issue_s = [&](int t, int j) -> bool {
          const int f = 2 * j;
          if (!wait_bar(&bars->kv_full[f % S], (f / S) & 1, args.fault, FAULT_FWD_KV)) return false;
          ptx::tc_fence_after();
          const uint32_t sKa = ptx::smem_u32(slot_addr(f));
          const uint32_t d_s = tmem + C::kColS + (uint32_t)t * kBN;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kSlabBytes + (kk & 3) * 32;
            const uint64_t a = ptx::sw128_desc(sQa + t * C::kTileBytes + off, 16, 1024);
            const uint64_t bd = ptx::sw128_desc(sKa + off, 16, 1024);
            ptx::mma_f16_ss(d_s, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(&bars->s_full[t]);
          return true;
        };
        // O_t += P_t(j) V(j); P_t in TMEM over the first 64 columns of S_t
        // (keys 2c, 2c+1 in column c).
        auto issue_pv = [&](int t, int j) -> bool {
          const int f = 2 * j + 1;
          if (!wait_bar(&bars->kv_full[f % S], (f / S) & 1, args.fault, FAULT_FWD_KV)) return false;
          if (!wait_bar(&bars->p_full[t], j & 1, args.fault, FAULT_FWD_P)) return false;
          ptx::tc_fence_after();
          const uint32_t sVa = ptx::smem_u32(slot_addr(f));
          const uint32_t a_p = tmem + C::kColS + (uint32_t)t * kBN;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t bd = ptx::sw128_desc(sVa + kk * 16 * 128, kSlabBytes, 1024);
            ptx::mma_f16_ts(tmem + C::kColO + (uint32_t)t * D, a_p + 8 * kk, bd, idesc_pv,
                            (j > 0 || kk > 0) ? 1u : 0u);
          }
          if (j + 1 == n_t[t]) ptx::mma_commit(&bars->o_done[t]);
          return true;
        };
        for (int t = 0; t < 2 && ok; ++t)
          if (n_t[t] > 0) ok = issue_s(t, 0);
        if (ok) ptx::mma_commit(&bars->kv_empty[0]);  // K(0): read by both S MMAs
        for (int j = 0; j < n_max && ok; ++j) {
          if (j < n_t[0] && !(ok = issue_pv(0, j))) break;
          if (j + 1 < n_t[0] && !(ok = issue_s(0, j + 1))) break;
          if (j < n_t[1] && !(ok = issue_pv(1, j))) break;
          ptx::mma_commit(&bars->kv_empty[(2 * j + 1) % S]);  // V(j): read by both P.V
          if (j + 1 < n_t[1] && !(ok = issue_s(1, j + 1))) break;
          if (j + 1 < n_max) ptx::mma_commit(&bars->kv_empty[(2 * j + 2) % S]);  // K(j+1)
        }
        // Drain: wait until every issued MMA has completed.
        ptx::mma_commit(&bars->drain);
        (void)wait_bar(&bars->drain, 0, nullptr, FAULT_FWD_DRAIN);
        if (!ok) record_fault(args.fault, FAULT_FWD_P);
      }
    }
  } else {
    // ------------------------- softmax warpgroups --------------------------
    ptx::setmaxnreg_inc<216>();
    const int t = (warp - 4) >> 2;           // query tile of this warpgroup
    const int row = (warp & 3) * 32 + lane;  // TMEM lane quarter = warp % 4
    const int r0 = q0 + t * kBM;             // first row of the tile
    const int qi = r0 + row;
    const int n_tiles = n_t[t];
    const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_s = C::kColS + (uint32_t)t * kBN;
    const uint32_t col_o = C::kColO + (uint32_t)t * D;
    const float qk_scale = (float)p.scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = !dead;
    for (int j = 0; j < n_tiles && ok; ++j) {
      // Warp-uniform outcome: the tcgen05.ld/st below are warp-collective.
      if (!__all_sync(0xffffffffu, wait_bar(&bars->s_full[t], j & 1, args.fault, FAULT_FWD_S))) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t r[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c)
        ptx::tmem_ld32(t_row + col_s + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(r + 32 * c));
      ptx::tmem_wait_ld();
      const int k0 = j * kBN;
      // Tiles away from the diagonal and the sequence end take the unmasked
      // branch (uniform for the warpgroup).
      const bool need_mask = (k0 + kBN > kv_end) || (p.is_causal && (int64_t)k0 + kBN - 1 > (int64_t)r0 + offset);
      const int64_t lim = p.is_causal ? (int64_t)qi + offset : (int64_t)kv_end - 1;
      // Row max of the (masked) raw scores, scaled once (scale > 0).
      float mx = -INFINITY;
      if (!need_mask) {
        float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
        for (int c = 0; c < kBN; c += 8) {
          m0 = ptx::max3(m0, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
          m1 = ptx::max3(m1, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
          m2 = ptx::max3(m2, __uint_as_float(r[c + 4]), __uint_as_float(r[c + 5]));
          m3 = ptx::max3(m3, __uint_as_float(r[c + 6]), __uint_as_float(r[c + 7]));
        }
        mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      } else {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const int key = k0 + c;
          if (key < kv_end && (int64_t)key <= lim) mx = fmaxf(mx, __uint_as_float(r[c]));
        }
      }
      mx = mx == -INFINITY ? mx : mx * qk_scale;
      const float m_new = fmaxf(m_run, mx);
      const bool rescale = m_new > m_run + kRescaleThreshold || (m_run == -INFINITY && m_new != -INFINITY);
      float factor = 1.f;
      if (rescale) {
        factor = m_run == -INFINITY ? 0.f : ptx::ex2(m_run - m_new);
        m_run = m_new;
        l_run *= factor;
      }
      const float safe = m_run == -INFINITY ? 0.f : m_run;
      // Dropout (kDrop): keep bits of the tile's 128 keys from the counter-based
      // generator the other kernels use (dropout.cuh); P.V sees p * keep / (1 - p),
      // the row sum l does not.
      uint32_t keep[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      if constexpr (kDrop) {
        const uint32_t bh = (uint32_t)(b * p.q_heads + h);
#pragma unroll
        for (int w = 0; w < 4; ++w) keep[w] = 0u;
#pragma unroll
        for (int j8 = 0; j8 < kBN / 8; ++j8)
          keep[j8 >> 2] |= dropout_keep8(args.drop, bh, (uint32_t)qi, (uint32_t)(k0 / 8 + j8)) << (8 * (j8 & 3));
      }
      auto dropped = [&](float pv, int c) -> float {
        if constexpr (kDrop) return (keep[c >> 5] >> (c & 31)) & 1u ? pv * args.drop.inv_keep_f : 0.f;
        return pv;
      };
      // P = exp2(s * scale * log2e - m) with packed f32x2 arithmetic: seven
      // element pairs in eight on MUFU ex2, the eighth on the FMA-pipe
      // polynomial (measured fastest of 0, 1, 2 and 3 pairs in eight on the
      // polynomial at the C5 shape); pairs packed with cvt.rn.
      uint32_t pk[kBN / 2];
      uint64_t sum2[2] = {ptx::f2pack(0.f, 0.f), ptx::f2pack(0.f, 0.f)};
      if (!need_mask) {
        const uint64_t sc2 = ptx::f2pack(qk_scale, qk_scale), ng2 = ptx::f2pack(-safe, -safe);
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          const uint64_t x2 = ptx::fma2(ptx::f2pack(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), sc2, ng2);
          uint64_t p2;
          if ((c & 14) != 14) {
            float x0, x1;
            ptx::f2unpack(x2, x0, x1);
            p2 = ptx::f2pack(ptx::ex2(x0), ptx::ex2(x1));
          } else {
            p2 = ptx::exp2_poly2(x2);
          }
          sum2[(c >> 1) & 1] = ptx::add2(sum2[(c >> 1) & 1], p2);
          float p0, p1;
          ptx::f2unpack(p2, p0, p1);
          p0 = dropped(p0, c);
          p1 = dropped(p1, c + 1);
          pk[c / 2] = kBF16 ? ptx::pack_bf16(p0, p1) : ptx::pack_f16(p0, p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          const int key = k0 + c;
          float p0 = ptx::ex2(fmaf(__uint_as_float(r[c]), qk_scale, -safe));
          float p1 = ptx::ex2(fmaf(__uint_as_float(r[c + 1]), qk_scale, -safe));
          p0 = (key < kv_end && (int64_t)key <= lim) ? p0 : 0.f;
          p1 = (key + 1 < kv_end && (int64_t)key + 1 <= lim) ? p1 : 0.f;
          sum2[0] = ptx::add2(sum2[0], ptx::f2pack(p0, p1));
          p0 = dropped(p0, c);
          p1 = dropped(p1, c + 1);
          pk[c / 2] = kBF16 ? ptx::pack_bf16(p0, p1) : ptx::pack_f16(p0, p1);
        }
      }
      {
        float a0, a1, b0, b1;
        ptx::f2unpack(sum2[0], a0, a1);
        ptx::f2unpack(sum2[1], b0, b1);
        l_run += (a0 + a1) + (b0 + b1);
      }
      // P_t(j) over the first 64 columns of S_t (those scores are in registers).
      ptx::tmem_st32(t_row + col_s, *reinterpret_cast<const uint32_t(*)[32]>(pk));
      ptx::tmem_st32(t_row + col_s + 32, *reinterpret_cast<const uint32_t(*)[32]>(pk + 32));
      // O_t holds P_t(0..j-1).V (S_t(j) was issued after the last of them):
      // rescale it in place before P_t(j).V accumulates into it.  Done after
      // the P store so that the scores' registers are free.  The TMEM round
      // trip is warp-collective, so the whole warp takes it when any row needs
      // it (factor 1 elsewhere).
      if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
        if (!rescale) factor = 1.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          ptx::tmem_ld32(t_row + col_o + 32 * c, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          ptx::tmem_st32(t_row + col_o + 32 * c, o);
        }
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[t]);
    }
    // Epilogue: O_t is final once its last P.V completed.
    if (ok && n_tiles > 0) ok = __all_sync(0xffffffffu, wait_bar(&bars->o_done[t], 0, args.fault, FAULT_FWD_O));
    ptx::tc_fence_after();
    const bool live_row = qi < p.q_len;
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
    T* orow = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
              (int64_t)qi * p.o.stride[2];
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t ra[32];
      if (n_tiles > 0 && ok) {
        ptx::tmem_ld32(t_row + col_o + 32 * c, ra);
        ptx::tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ra[e] = 0u;
      }
      if (live_row) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          float f[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) f[u] = __uint_as_float(ra[e + u]) * inv;
          uint4 v;
          if (kBF16) {
            v = make_uint4(ptx::pack_bf16(f[0], f[1]), ptx::pack_bf16(f[2], f[3]), ptx::pack_bf16(f[4], f[5]),
                           ptx::pack_bf16(f[6], f[7]));
          } else {
            v = make_uint4(ptx::pack_f16(f[0], f[1]), ptx::pack_f16(f[2], f[3]), ptx::pack_f16(f[4], f[5]),
                           ptx::pack_f16(f[6], f[7]));
          }
          *reinterpret_cast<uint4*>(orow + 32 * c + e) = v;
        }
      }
    }
    if (live_row && p.lse)
      reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] +
                                      (int64_t)qi * p.lse_stride[2]] =
          l_run > 0.f ? (m_run + __log2f(l_run)) * kLn2 : -INFINITY;
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int D, bool BF16>
static cudaError_t launch_pair(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                               const PairArgs& a, cudaStream_t st) {
  auto kern = a.drop.p > 0.f ? tc_fwd_pair_kernel<D, BF16, true> : tc_fwd_pair_kernel<D, BF16, false>;
  cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(kern), PairCfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.n_units, a.p.q_heads, a.p.batch);
  kern<<<grid, 384, PairCfg<D>::kSmem, st>>>(mq, mk, mv, a);
  return cudaGetLastError();
}

cudaError_t tc_forward_pair(const ts_attn_params& p, const CUtensorMap& mq, const CUtensorMap& mk,
                            const CUtensorMap& mv, uint32_t* fault, cudaStream_t st, const DropoutArgs* drop) {
  PairArgs a;
  a.p = p;
  a.n_units = ceil_div(p.q_len, 2 * kBM);
  a.fault = fault;
  a.drop = drop ? *drop : DropoutArgs{};
  const bool bf = p.dtype == TS_BF16;
  if (p.head_dim == 64) return bf ? launch_pair<64, true>(mq, mk, mv, a, st) : launch_pair<64, false>(mq, mk, mv, a, st);
  return bf ? launch_pair<128, true>(mq, mk, mv, a, st) : launch_pair<128, false>(mq, mk, mv, a, st);
}

}  // namespace tsa
