// Causal / full prefill attention forward on the 5th-generation tensor cores
// (tcgen05) for bf16 / f16 inputs with D = Dv in {64, 128}.
//
// Replaces the dense / streaming forwards of tensorsmith's nn/attention.py
// (:132-145, :175-198) and fills the vendor "native" slot (:146-174) on CUDA:
// the same online-softmax recurrence (running max, running sum, rescaled
// accumulator; output a/l; LSE = m + log l), computed tile by tile without
// materialising P in HBM and skipping key tiles the causal rule hides.
//
// One CTA = one 128-row query tile of one (batch, head).  Warp roles:
//   warp 0   TMA producer: Q once, then K/V 128-key tiles into 2-stage rings
//            (separate K and V rings so K(j+2) can land while P(j).V(j) runs)
//   warp 1   MMA issuer (one thread): S = Q K^T into a double-buffered TMEM S,
//            then O_A += P_A V[0:64) and O_B += P_B V[64:128) into two TMEM
//            accumulators, with P_A / P_B read from TMEM (A operand in tensor
//            memory); completion signalled with tcgen05.commit
//   warp 2   TMEM allocator (512 columns: S0 | S1 | O_A | O_B)
//   warps 4-7 and 8-11: two softmax warpgroups over the same 128 rows; group
//            A owns keys [0, 64) of every tile, group B keys [64, 128).  Thread
//            r of a group owns query row r (TMEM lane r) and runs an
//            independent exp2-domain online softmax over its key half (its own
//            running max and sum, lazy rescaling of its own O accumulator when
//            the max grows by more than 2^8), writing P (bf16/f16 pairs) back
//            into TMEM over the S columns it just read, where the P.V MMA takes
//            it as its A operand (no shared-memory round trip for P).  The
//            halves never synchronise in
//            the key loop; the epilogue merges them once:
//            O = (O_A 2^(m_A-m) + O_B 2^(m_B-m)) / (l_A 2^(m_A-m) + l_B 2^(m_B-m)).
//            Two warps per scheduler hide the TMEM-load and MUFU latencies that
//            a single warpgroup of 128-key rows leaves exposed.
// tc_fwd_persistent_kernel below runs the same roles over several query tiles
// per CTA for short causal rows.
// Shared-memory operands use the canonical 128-byte-swizzle layouts: Q and K
// are K-major (8-row x 128-byte atoms, 1024 B apart); V is read MN-major
// (64-channel blocks 16 KB apart, 8-key groups 1024 B apart).  No TMA load
// uses cluster multicast.
#include <cstdlib>
#include <cstring>
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
constexpr uint32_t kFaultSmemAlign = 0x108;  // dynamic shared memory needed more alignment slack

template <int D> struct Cfg {
  static constexpr int kSlabs = D / 64;
  static constexpr int kStages = 3;
  static constexpr int kTileBytes = kSlabs * kSlabBytes;  // one 128-row Q/K/V tile
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffRed = kOffV + kStages * kTileBytes;  // epilogue exchange [half][row][m, l]
  static constexpr int kOffBar = kOffRed + 2 * 128 * 2 * 4;
  static constexpr int kBarBytes = 256;
  // Alignment slack for the 1024-byte-aligned tile base: D=128 fills the
  // 227 KB opt-in limit exactly, so it keeps 768 bytes and the kernel refuses
  // to run (fault word, no access) if the dynamic window needs more.
  static constexpr int kSlack = D == 128 ? 768 : 1024;
  static constexpr int kSmem = kOffBar + kBarBytes + kSlack;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColS = 0;     // two 128-column S buffers
  static constexpr uint32_t kColO = 256;   // O_A (D columns), then O_B (D columns)
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[3], v_empty[3];
  uint64_t s_full[2];
  uint64_t p_full[2];  // per key half
  uint64_t o_done[2];
  uint64_t epi;        // both halves posted their (m, l)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Barriers of the persistent kernel: those of Bars plus the hand-over of Q and
// of the O accumulators (and of the epilogue exchange) from one query tile to the next.
struct PBars {
  uint64_t q_full, q_empty;
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[3], v_empty[3];
  uint64_t s_full[2];
  uint64_t p_full[2];  // per key half
  uint64_t o_done[2];
  uint64_t o_free;     // the epilogue read both O accumulators
  uint64_t epi;        // both halves posted their (m, l)
  uint64_t red_free;   // both halves read the exchange
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct TcFwdArgs {
  ts_attn_params p;
  int n_q_tiles;
  int half_x;   // ceil(n_q_tiles / 2): query-tile pairs per (batch, head)
  int n_units;  // batch * heads * half_x
  uint32_t* fault;
  DropoutArgs drop;  // used by the kDrop instantiation only
};

}  // namespace

template <int D, bool kBF16, bool kDrop>
__global__ void __launch_bounds__(384, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, TcFwdArgs args) {
  using C = Cfg<D>;
  const ts_attn_params& p = args.p;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t pad = (1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad > (uint32_t)C::kSlack) {  // uniform for the CTA: nothing initialised yet
    if (threadIdx.x == 0) record_fault(args.fault, kFaultSmemAlign);
    return;
  }
  unsigned char* smem = smem_raw + pad;
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  unsigned char* sQ = smem + C::kOffQ;
  unsigned char* sK = smem + C::kOffK;
  unsigned char* sV = smem + C::kOffV;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_tile = args.n_q_tiles - 1 - (int)blockIdx.x;  // longest causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.q_heads / p.kv_heads);

  // Visible key range of this tile.
  int kv_end = p.kv_len;
  int64_t offset = p.causal_offset;
  if (p.kv_lens) {
    kv_end = min(kv_end, max(0, p.kv_lens[b]));
    offset = (int64_t)kv_end - p.q_len;
  }
  const int q0 = q_tile * kBM;
  const int q_last = min(q0 + kBM - 1, p.q_len - 1);
  int kv_lim = kv_end;
  if (p.is_causal) kv_lim = (int)i64max(0, i64min(kv_end, (int64_t)q_last + offset + 1));
  const int n_tiles = ceil_div(kv_lim, kBN);
  const bool dead = fault_set(args.fault);

  if (threadIdx.x == 0) {
    ptx::mbar_init(&bars->q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&bars->k_full[s], 1);
      ptx::mbar_init(&bars->k_empty[s], 1);
      ptx::mbar_init(&bars->v_full[s], 1);
      ptx::mbar_init(&bars->v_empty[s], 1);
    }
    ptx::mbar_init(&bars->s_full[0], 1);
    ptx::mbar_init(&bars->s_full[1], 1);
    for (int hf = 0; hf < 2; ++hf) {
      ptx::mbar_init(&bars->p_full[hf], 4);
      ptx::mbar_init(&bars->o_done[hf], 1);
    }
    ptx::mbar_init(&bars->epi, 8);
    ptx::mbar_init(&bars->drain, 1);
    bars->abort = 0;
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

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0 && n_tiles > 0 && !dead) {
      ptx::prefetch_tensormap(&tm_q);
      ptx::prefetch_tensormap(&tm_k);
      ptx::prefetch_tensormap(&tm_v);
      ptx::mbar_expect_tx(&bars->q_full, C::kTileBytes);
      for (int s = 0; s < C::kSlabs; ++s)
        ptx::tma_load_4d(sQ + s * kSlabBytes, &tm_q, 64 * s, q0, h, b, &bars->q_full);
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % C::kStages;
        const uint32_t ph = ((j / C::kStages) - 1) & 1;
        if (j >= C::kStages && !wait_bar(&bars->k_empty[s], ph, args.fault, FAULT_FWD_EMPTY)) break;
        ptx::mbar_expect_tx(&bars->k_full[s], C::kTileBytes);
        for (int sl = 0; sl < C::kSlabs; ++sl)
          ptx::tma_load_4d(sK + (s * C::kSlabs + sl) * kSlabBytes, &tm_k, 64 * sl, j * kBN, hk, b,
                           &bars->k_full[s]);
        k_issued = j + 1;
        if (j >= C::kStages && !wait_bar(&bars->v_empty[s], ph, args.fault, FAULT_FWD_EMPTY)) break;
        ptx::mbar_expect_tx(&bars->v_full[s], C::kTileBytes);
        for (int sl = 0; sl < C::kSlabs; ++sl)
          ptx::tma_load_4d(sV + (s * C::kSlabs + sl) * kSlabBytes, &tm_v, 64 * sl, j * kBN, hk, b,
                           &bars->v_full[s]);
        v_issued = j + 1;
      }
      // Drain: every issued copy must have landed before shared memory is released.
      (void)wait_bar(&bars->q_full, 0, nullptr, FAULT_FWD_DRAIN);
      for (int j = max(0, k_issued - C::kStages); j < k_issued; ++j)
        (void)wait_bar(&bars->k_full[j % C::kStages], (j / C::kStages) & 1, nullptr, FAULT_FWD_DRAIN);
      for (int j = max(0, v_issued - C::kStages); j < v_issued; ++j)
        (void)wait_bar(&bars->v_full[j % C::kStages], (j / C::kStages) & 1, nullptr, FAULT_FWD_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0 && n_tiles > 0 && !dead) {
      constexpr uint32_t idesc_qk = ptx::idesc_f16(kBF16, kBM, kBN, false, false);
      const uint32_t sQa = ptx::smem_u32(sQ), sKa = ptx::smem_u32(sK), sVa = ptx::smem_u32(sV);
      bool ok = wait_bar(&bars->q_full, 0, args.fault, FAULT_FWD_Q);
      ptx::tc_fence_after();
      constexpr uint32_t idesc_pv = ptx::idesc_f16(kBF16, kBM, D, false, true);
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj % C::kStages;
        if (!wait_bar(&bars->v_full[s], (jj / C::kStages) & 1, args.fault, FAULT_FWD_KV)) return false;
        // Key half hf: P_hf (slab hf) times V keys [64 hf, 64 hf + 64) into O_hf.
        for (int hf = 0; hf < 2; ++hf) {
          if (!wait_bar(&bars->p_full[hf], jj & 1, args.fault, FAULT_FWD_P)) return false;
          ptx::tc_fence_after();
          // P_hf lives in TMEM over the first 32 columns of its S(jj) half (bf16x2 per column).
          const uint32_t a_p = tmem + C::kColS + (uint32_t)(jj & 1) * kBN + hf * (kBN / 2);
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {
            const int kk = hf * 4 + kq;
            const uint64_t bd =
                ptx::sw128_desc(sVa + s * C::kTileBytes + kk * 16 * 128, kSlabBytes, 1024);
            ptx::mma_f16_ts(tmem + C::kColO + hf * D, a_p + 8 * kq, bd, idesc_pv, (jj > 0 || kq > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&bars->o_done[hf]);
        }
        ptx::mma_commit(&bars->v_empty[s]);
        return true;
      };
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j % C::kStages;
        if (!wait_bar(&bars->k_full[s], (j / C::kStages) & 1, args.fault, FAULT_FWD_KV)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_s = tmem + C::kColS + (uint32_t)(j & 1) * kBN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kSlabBytes + (kk & 3) * 32;
          const uint64_t a = ptx::sw128_desc(sQa + off, 16, 1024);
          const uint64_t bd = ptx::sw128_desc(sKa + s * C::kTileBytes + off, 16, 1024);
          ptx::mma_f16_ss(d_s, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&bars->s_full[j & 1]);
        ptx::mma_commit(&bars->k_empty[s]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok) ok = issue_pv(n_tiles - 1);
      // Drain: wait until every issued MMA has completed.
      ptx::mma_commit(&bars->drain);
      (void)wait_bar(&bars->drain, 0, nullptr, FAULT_FWD_DRAIN);
      if (!ok) atomicExch(&bars->abort, 1);
    }
  } else if (warp >= 4) {
    // ------------------------- softmax warpgroups --------------------------
    const int half = (warp - 4) >> 2;           // 0: keys [0, 64) of a tile, 1: keys [64, 128)
    const int row = (warp & 3) * 32 + lane;     // TMEM lane quarter = warp % 4
    const int qi = q0 + row;
    const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_o = C::kColO + (uint32_t)half * D;
    const float qk_scale = (float)p.scale * kLog2e;
    constexpr int kHN = kBN / 2;  // keys per half
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = !dead;
    for (int j = 0; j < n_tiles && ok; ++j) {
      // Warp-uniform outcome: the tcgen05.ld/st below are warp-collective.
      if (!__all_sync(0xffffffffu, wait_bar(&bars->s_full[j & 1], (j >> 1) & 1, args.fault, FAULT_FWD_S))) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      // The 64 raw scores of this row's key half in registers (two loads, one wait).
      uint32_t r[kHN];
#pragma unroll
      for (int c = 0; c < kHN / 32; ++c)
        ptx::tmem_ld32(t_row + C::kColS + (uint32_t)(j & 1) * kBN + half * kHN + 32 * c,
                       *reinterpret_cast<uint32_t(*)[32]>(r + 32 * c));
      ptx::tmem_wait_ld();
      const int k0 = j * kBN + half * kHN;
      const bool need_mask = (k0 + kHN > kv_end) || (p.is_causal && (int64_t)k0 + kHN - 1 > (int64_t)q0 + offset);
      const int64_t lim = p.is_causal ? (int64_t)qi + offset : (int64_t)kv_end - 1;
      // Row max of the (masked) raw scores, scaled once (scale > 0).  Halves
      // away from the diagonal and the sequence end take the unmasked branch
      // (warp-uniform).
      float mx = -INFINITY;
      if (!need_mask) {
        float m0 = -INFINITY, m1 = -INFINITY;  // two chains halve the dependent-max latency
#pragma unroll
        for (int c = 0; c < kHN; c += 4) {
          m0 = ptx::max3(m0, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
          m1 = ptx::max3(m1, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
        }
        mx = fmaxf(m0, m1);
      } else {
#pragma unroll
        for (int c = 0; c < kHN; ++c) {
          const int key = k0 + c;
          if (key < kv_end && (int64_t)key <= lim) mx = fmaxf(mx, __uint_as_float(r[c]));
        }
      }
      mx = mx == -INFINITY ? mx : mx * qk_scale;
      const float m_new = fmaxf(m_run, mx);
      const bool rescale = m_new > m_run + kRescaleThreshold ||
                           (m_run == -INFINITY && m_new != -INFINITY);
      float factor = 1.f;
      if (rescale) {
        factor = m_run == -INFINITY ? 0.f : ptx::ex2(m_run - m_new);
        m_run = m_new;
        l_run *= factor;
      }
      const float safe = m_run == -INFINITY ? 0.f : m_run;
      // P = exp2(s * scale * log2e - m) with packed f32x2 arithmetic; seven
      // element pairs in eight go through MUFU ex2 and the eighth through the
      // FMA-pipe polynomial (the split measured fastest at the C5 shape: the
      // polynomial costs about five times the issue slots of MUFU, and MUFU
      // alone would take as long as the tile's MMAs); pairs are packed with
      // cvt.rn (measured 1.4 % faster than integer rounding at that shape).
      uint32_t pk[kHN / 2];
      uint64_t sum2[2] = {ptx::f2pack(0.f, 0.f), ptx::f2pack(0.f, 0.f)};
      // Dropout (kDrop): keep bits of this half's 64 keys, from the counter-based
      // generator the generic kernels use (dropout.cuh); P.V sees p * keep / (1 - p),
      // the row sum l does not.
      uint32_t keep[2] = {0xffffffffu, 0xffffffffu};
      if constexpr (kDrop) {
        const uint32_t bh = (uint32_t)(b * p.q_heads + h);
        keep[0] = keep[1] = 0u;
#pragma unroll
        for (int j8 = 0; j8 < kHN / 8; ++j8)
          keep[j8 >> 2] |= dropout_keep8(args.drop, bh, (uint32_t)qi, (uint32_t)(k0 / 8 + j8)) << (8 * (j8 & 3));
      }
      auto dropped = [&](float pv, int c) -> float {
        if constexpr (kDrop) return (keep[c >> 5] >> (c & 31)) & 1u ? pv * args.drop.inv_keep_f : 0.f;
        return pv;
      };
      if (!need_mask) {
        const uint64_t sc2 = ptx::f2pack(qk_scale, qk_scale), ng2 = ptx::f2pack(-safe, -safe);
#pragma unroll
        for (int c = 0; c < kHN; c += 2) {
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
        for (int c = 0; c < kHN; c += 2) {
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
      // P(j) into TMEM over the first 32 columns of this half's S(j) (already in
      // registers); P(j).V(j) reads it from there, and S(j+2) only overwrites it
      // after that MMA (one issuing thread, executed in order).
      ptx::tmem_st32(t_row + C::kColS + (uint32_t)(j & 1) * kBN + half * kHN,
                     pk);
      ptx::tmem_wait_st();
      // This half's O accumulator may be rescaled once P(j-1).V(j-1) of the half completed.
      if (j >= 1 &&
          !__all_sync(0xffffffffu, wait_bar(&bars->o_done[half], (j - 1) & 1, args.fault, FAULT_FWD_O))) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      // The rescale decision is per row; the TMEM round trip is warp-collective,
      // so the whole warp takes it when any row needs it (factor 1 elsewhere).
      if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
        if (!rescale) factor = 1.f;
        uint32_t o[32];
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          ptx::tmem_ld32(t_row + col_o + 32 * c, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          ptx::tmem_st32(t_row + col_o + 32 * c, o);
        }
        ptx::tmem_wait_st();
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[half]);
    }
    // Epilogue: both O accumulators must be final (each thread reads both).
    if (ok && n_tiles > 0) {
      const uint32_t ph = (n_tiles - 1) & 1;
      ok = __all_sync(0xffffffffu, wait_bar(&bars->o_done[0], ph, args.fault, FAULT_FWD_O) &&
                                       wait_bar(&bars->o_done[1], ph, args.fault, FAULT_FWD_O));
    }
    ptx::tc_fence_after();
    // Exchange (m, l) with the other half of the row, once.
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
    red[(half * 128 + row) * 2 + 0] = m_run;
    red[(half * 128 + row) * 2 + 1] = l_run;
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&bars->epi);
    ok = __all_sync(0xffffffffu, ok && wait_bar(&bars->epi, 0, args.fault, FAULT_FWD_O));
    const float m_oth = red[((1 - half) * 128 + row) * 2 + 0];
    const float l_oth = red[((1 - half) * 128 + row) * 2 + 1];
    const float m_a = half == 0 ? m_run : m_oth, l_a = half == 0 ? l_run : l_oth;
    const float m_b = half == 0 ? m_oth : m_run, l_b = half == 0 ? l_oth : l_run;
    const float m_all = fmaxf(m_a, m_b);
    const float m_safe = m_all == -INFINITY ? 0.f : m_all;
    const float f_a = m_a == -INFINITY ? 0.f : ptx::ex2(m_a - m_safe);
    const float f_b = m_b == -INFINITY ? 0.f : ptx::ex2(m_b - m_safe);
    const float l_all = l_a * f_a + l_b * f_b;
    const bool live_row = qi < p.q_len;
    const float inv = l_all > 0.f ? 1.f / l_all : 0.f;
    const float w_a = f_a * inv, w_b = f_b * inv;
    using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
    T* orow = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
              (int64_t)qi * p.o.stride[2];
    // This thread writes output channels [half * D/2, half * D/2 + D/2).
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      const uint32_t col = (uint32_t)(half * (D / 2) + 32 * c);
      uint32_t ra[32], rb[32];
      if (n_tiles > 0 && ok) {
        ptx::tmem_ld32(t_row + C::kColO + col, ra);
        ptx::tmem_ld32(t_row + C::kColO + D + col, rb);
        ptx::tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ra[e] = rb[e] = 0u;
      }
      if (live_row) {
        float f[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(ra[e]) * w_a + __uint_as_float(rb[e]) * w_b;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 v;
          if (kBF16) {
            v = make_uint4(ptx::pack_bf16(f[e], f[e + 1]), ptx::pack_bf16(f[e + 2], f[e + 3]),
                           ptx::pack_bf16(f[e + 4], f[e + 5]), ptx::pack_bf16(f[e + 6], f[e + 7]));
          } else {
            v = make_uint4(ptx::pack_f16(f[e], f[e + 1]), ptx::pack_f16(f[e + 2], f[e + 3]),
                           ptx::pack_f16(f[e + 4], f[e + 5]), ptx::pack_f16(f[e + 6], f[e + 7]));
          }
          *reinterpret_cast<uint4*>(orow + col + e) = v;
        }
      }
    }
    if (live_row && p.lse && half == 0)
      reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] + (int64_t)qi * p.lse_stride[2]] =
          l_all > 0.f ? (m_all + __log2f(l_all)) * kLn2 : -INFINITY;
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Persistent variant of the same pipeline, for short causal rows (see
// use_persistent): one CTA per SM takes work units u = blockIdx.x,
// blockIdx.x + gridDim.x, ... in (batch, head)-major order, so the CTAs running
// at once share K/V in L2.  A unit is the longest and the shortest remaining
// query tile of one (batch, head) (tiles X-1-t and t), so every unit of a
// causal problem carries X + 1 key tiles and the static schedule is balanced.
// The warp roles are those of tc_fwd_kernel; their pipelines run on across
// query tiles: global key-tile counters keep the ring stages and barrier
// phases going, the producer loads the next tile's Q as soon as the last S
// MMA of the current one completed (q_empty), and the MMA warp computes the
// next tile's first S blocks while the softmax warps run the epilogue; the
// next tile's first P.V, which overwrites O, waits for that epilogue (o_free).
// Query tiles with no visible key touch no barrier in any role.
template <int D, bool kBF16, bool kDrop>
__global__ void __launch_bounds__(384, 1)
    tc_fwd_persistent_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, TcFwdArgs args) {
  using C = Cfg<D>;
  const ts_attn_params& p = args.p;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t pad = (1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad > (uint32_t)C::kSlack) {  // uniform for the CTA: nothing initialised yet
    if (threadIdx.x == 0) record_fault(args.fault, kFaultSmemAlign);
    return;
  }
  unsigned char* smem = smem_raw + pad;
  PBars* bars = reinterpret_cast<PBars*>(smem + C::kOffBar);
  unsigned char* sQ = smem + C::kOffQ;
  unsigned char* sK = smem + C::kOffK;
  unsigned char* sV = smem + C::kOffV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool dead = fault_set(args.fault);

  if (threadIdx.x == 0) {
    ptx::mbar_init(&bars->q_full, 1);
    ptx::mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&bars->k_full[s], 1);
      ptx::mbar_init(&bars->k_empty[s], 1);
      ptx::mbar_init(&bars->v_full[s], 1);
      ptx::mbar_init(&bars->v_empty[s], 1);
    }
    ptx::mbar_init(&bars->s_full[0], 1);
    ptx::mbar_init(&bars->s_full[1], 1);
    for (int hf = 0; hf < 2; ++hf) {
      ptx::mbar_init(&bars->p_full[hf], 4);
      ptx::mbar_init(&bars->o_done[hf], 1);
    }
    ptx::mbar_init(&bars->o_free, 8);
    ptx::mbar_init(&bars->epi, 8);
    ptx::mbar_init(&bars->red_free, 8);
    ptx::mbar_init(&bars->drain, 1);
    bars->abort = 0;
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

  // This CTA's query tiles, in the same order for every role: work units u =
  // blockIdx.x, blockIdx.x + gridDim.x, ...; unit u = the longest and the
  // shortest remaining query tile (X-1-t and t) of one (batch, head), so all
  // units of a causal problem carry the same number of key tiles.  Tiles with
  // no visible key touch no barrier in any role.
  const int n_units = args.n_units, half_x = args.half_x, nq = args.n_q_tiles;
#define TS_FOR_EACH_QTILE(...)                                                                    \
  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {                                          \
    const int pair_ = u / half_x, t_ = u % half_x;                                                 \
    for (int sub_ = 0; sub_ < 2; ++sub_) {                                                         \
      const int qt = sub_ == 0 ? nq - 1 - t_ : t_;                                                 \
      if (sub_ == 1 && qt == nq - 1 - t_) break;                                                   \
      const int h = pair_ % p.q_heads, b = pair_ / p.q_heads;                                      \
      const int hk = h / (p.q_heads / p.kv_heads);                                                 \
      int kv_end = p.kv_len;                                                                       \
      int64_t offset = p.causal_offset;                                                            \
      if (p.kv_lens) {                                                                             \
        kv_end = min(kv_end, max(0, p.kv_lens[b]));                                                \
        offset = (int64_t)kv_end - p.q_len;                                                        \
      }                                                                                            \
      const int q0 = qt * kBM;                                                                     \
      const int q_last = min(q0 + kBM - 1, p.q_len - 1);                                           \
      int kv_lim = kv_end;                                                                         \
      if (p.is_causal) kv_lim = (int)i64max(0, i64min(kv_end, (int64_t)q_last + offset + 1));     \
      const int n_tiles = ceil_div(kv_lim, kBN);                                                   \
      (void)hk;                                                                                    \
      __VA_ARGS__                                                                                  \
    }                                                                                              \
  }

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0 && !dead) {
      ptx::prefetch_tensormap(&tm_q);
      ptx::prefetch_tensormap(&tm_k);
      ptx::prefetch_tensormap(&tm_v);
      int gk = 0, iq = 0, k_issued = 0, v_issued = 0;
      bool ok = true;
      TS_FOR_EACH_QTILE({
        if (n_tiles > 0 && ok) {
          // Q of the previous tile is free once that tile's last S MMA completed.
          if (iq >= 1 && !wait_bar(&bars->q_empty, (iq - 1) & 1, args.fault, FAULT_FWD_EMPTY)) {
            ok = false;
          } else {
            ptx::mbar_expect_tx(&bars->q_full, C::kTileBytes);
            for (int s = 0; s < C::kSlabs; ++s)
              ptx::tma_load_4d(sQ + s * kSlabBytes, &tm_q, 64 * s, q0, h, b, &bars->q_full);
            for (int j = 0; j < n_tiles && ok; ++j) {
              const int g = gk + j;
              const int s = g % C::kStages;
              const uint32_t ph = ((g / C::kStages) - 1) & 1;
              if (g >= C::kStages && !wait_bar(&bars->k_empty[s], ph, args.fault, FAULT_FWD_EMPTY)) {
                ok = false;
                break;
              }
              ptx::mbar_expect_tx(&bars->k_full[s], C::kTileBytes);
              for (int sl = 0; sl < C::kSlabs; ++sl)
                ptx::tma_load_4d(sK + (s * C::kSlabs + sl) * kSlabBytes, &tm_k, 64 * sl, j * kBN, hk, b,
                                 &bars->k_full[s]);
              k_issued = g + 1;
              if (g >= C::kStages && !wait_bar(&bars->v_empty[s], ph, args.fault, FAULT_FWD_EMPTY)) {
                ok = false;
                break;
              }
              ptx::mbar_expect_tx(&bars->v_full[s], C::kTileBytes);
              for (int sl = 0; sl < C::kSlabs; ++sl)
                ptx::tma_load_4d(sV + (s * C::kSlabs + sl) * kSlabBytes, &tm_v, 64 * sl, j * kBN, hk, b,
                                 &bars->v_full[s]);
              v_issued = g + 1;
            }
            gk += n_tiles;
            ++iq;
          }
        }
      })
      // Drain: every issued copy must have landed before shared memory is released.
      if (iq > 0) (void)wait_bar(&bars->q_full, (iq - 1) & 1, nullptr, FAULT_FWD_DRAIN);
      for (int g = max(0, k_issued - C::kStages); g < k_issued; ++g)
        (void)wait_bar(&bars->k_full[g % C::kStages], (g / C::kStages) & 1, nullptr, FAULT_FWD_DRAIN);
      for (int g = max(0, v_issued - C::kStages); g < v_issued; ++g)
        (void)wait_bar(&bars->v_full[g % C::kStages], (g / C::kStages) & 1, nullptr, FAULT_FWD_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0 && !dead) {
      constexpr uint32_t idesc_qk = ptx::idesc_f16(kBF16, kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = ptx::idesc_f16(kBF16, kBM, D, false, true);
      const uint32_t sQa = ptx::smem_u32(sQ), sKa = ptx::smem_u32(sK), sVa = ptx::smem_u32(sV);
      bool ok = true;
      // P(g).V(g) of global key tile g; `first` = the first tile of its query tile,
      // whose MMAs overwrite O once the previous query tile's epilogue read it.
      auto issue_pv = [&](int gg, bool first, int iq_of) -> bool {
        const int s = gg % C::kStages;
        if (first && iq_of >= 1 && !wait_bar(&bars->o_free, (iq_of - 1) & 1, args.fault, FAULT_FWD_O)) return false;
        if (!wait_bar(&bars->v_full[s], (gg / C::kStages) & 1, args.fault, FAULT_FWD_KV)) return false;
        for (int hf = 0; hf < 2; ++hf) {
          if (!wait_bar(&bars->p_full[hf], gg & 1, args.fault, FAULT_FWD_P)) return false;
          ptx::tc_fence_after();
          const uint32_t a_p = tmem + C::kColS + (uint32_t)(gg & 1) * kBN + hf * (kBN / 2);
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {
            const int kk = hf * 4 + kq;
            const uint64_t bd = ptx::sw128_desc(sVa + s * C::kTileBytes + kk * 16 * 128, kSlabBytes, 1024);
            ptx::mma_f16_ts(tmem + C::kColO + hf * D, a_p + 8 * kq, bd, idesc_pv, (!first || kq > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&bars->o_done[hf]);
        }
        ptx::mma_commit(&bars->v_empty[s]);
        return true;
      };
      int gk = 0, iq = 0;
      int pend_g = -1, pend_iq = 0;
      bool pend_first = false;
      TS_FOR_EACH_QTILE({
        if (n_tiles > 0 && ok) {
          // Finish the previous query tile (its last P.V) before waiting for this one's Q.
          if (pend_g >= 0) {
            if (!issue_pv(pend_g, pend_first, pend_iq)) ok = false;
            pend_g = -1;
          }
          if (ok && !wait_bar(&bars->q_full, iq & 1, args.fault, FAULT_FWD_Q)) ok = false;
          ptx::tc_fence_after();
          for (int j = 0; j < n_tiles && ok; ++j) {
            const int g = gk + j;
            const int s = g % C::kStages;
            if (!wait_bar(&bars->k_full[s], (g / C::kStages) & 1, args.fault, FAULT_FWD_KV)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t d_s = tmem + C::kColS + (uint32_t)(g & 1) * kBN;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * kSlabBytes + (kk & 3) * 32;
              const uint64_t a = ptx::sw128_desc(sQa + off, 16, 1024);
              const uint64_t bd = ptx::sw128_desc(sKa + s * C::kTileBytes + off, 16, 1024);
              ptx::mma_f16_ss(d_s, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
            }
            ptx::mma_commit(&bars->s_full[g & 1]);
            ptx::mma_commit(&bars->k_empty[s]);
            if (j == n_tiles - 1) ptx::mma_commit(&bars->q_empty);  // Q read by every S of this tile
            if (pend_g >= 0 && !issue_pv(pend_g, pend_first, pend_iq)) {
              ok = false;
              break;
            }
            pend_g = g;
            pend_first = j == 0;
            pend_iq = iq;
          }
          gk += n_tiles;
          ++iq;
        }
      })
      if (ok && pend_g >= 0) ok = issue_pv(pend_g, pend_first, pend_iq);
      // Drain: wait until every issued MMA has completed.
      ptx::mma_commit(&bars->drain);
      (void)wait_bar(&bars->drain, 0, nullptr, FAULT_FWD_DRAIN);
      if (!ok) atomicExch(&bars->abort, 1);
    }
  } else if (warp >= 4) {
    // ------------------------- softmax warpgroups --------------------------
    const int half = (warp - 4) >> 2;           // 0: keys [0, 64) of a tile, 1: keys [64, 128)
    const int row = (warp & 3) * 32 + lane;     // TMEM lane quarter = warp % 4
    const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_o = C::kColO + (uint32_t)half * D;
    const float qk_scale = (float)p.scale * kLog2e;
    constexpr int kHN = kBN / 2;  // keys per half
    using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
    bool ok = !dead;
    int gk = 0, iq = 0;
    TS_FOR_EACH_QTILE({
      const int qi = q0 + row;
      const bool live_row = qi < p.q_len;
      T* orow = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
                (int64_t)qi * p.o.stride[2];
      if (n_tiles == 0) {
        // No visible key: zero output, LSE -inf (nn/attention.py:126-127, 194-196).
        if (live_row) {
#pragma unroll
          for (int c = 0; c < D / 2; c += 8)
            *reinterpret_cast<uint4*>(orow + half * (D / 2) + c) = make_uint4(0u, 0u, 0u, 0u);
          if (p.lse && half == 0)
            reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] +
                                            (int64_t)qi * p.lse_stride[2]] = -INFINITY;
        }
      } else if (ok) {
        float m_run = -INFINITY, l_run = 0.f;
        for (int j = 0; j < n_tiles && ok; ++j) {
          const int g = gk + j;
          // Warp-uniform outcome: the tcgen05.ld/st below are warp-collective.
          if (!__all_sync(0xffffffffu, wait_bar(&bars->s_full[g & 1], (g >> 1) & 1, args.fault, FAULT_FWD_S))) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          // The 64 raw scores of this row's key half in registers (two loads, one wait).
          uint32_t r[kHN];
    #pragma unroll
          for (int c = 0; c < kHN / 32; ++c)
            ptx::tmem_ld32(t_row + C::kColS + (uint32_t)(g & 1) * kBN + half * kHN + 32 * c,
                           *reinterpret_cast<uint32_t(*)[32]>(r + 32 * c));
          ptx::tmem_wait_ld();
          const int k0 = j * kBN + half * kHN;
          const bool need_mask = (k0 + kHN > kv_end) || (p.is_causal && (int64_t)k0 + kHN - 1 > (int64_t)q0 + offset);
          const int64_t lim = p.is_causal ? (int64_t)qi + offset : (int64_t)kv_end - 1;
          // Row max of the (masked) raw scores, scaled once (scale > 0).  Halves
          // away from the diagonal and the sequence end take the unmasked branch
          // (warp-uniform).
          float mx = -INFINITY;
          if (!need_mask) {
            float m0 = -INFINITY, m1 = -INFINITY;  // two chains halve the dependent-max latency
    #pragma unroll
            for (int c = 0; c < kHN; c += 4) {
              m0 = ptx::max3(m0, __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
              m1 = ptx::max3(m1, __uint_as_float(r[c + 2]), __uint_as_float(r[c + 3]));
            }
            mx = fmaxf(m0, m1);
          } else {
    #pragma unroll
            for (int c = 0; c < kHN; ++c) {
              const int key = k0 + c;
              if (key < kv_end && (int64_t)key <= lim) mx = fmaxf(mx, __uint_as_float(r[c]));
            }
          }
          mx = mx == -INFINITY ? mx : mx * qk_scale;
          const float m_new = fmaxf(m_run, mx);
          const bool rescale = m_new > m_run + kRescaleThreshold ||
                               (m_run == -INFINITY && m_new != -INFINITY);
          float factor = 1.f;
          if (rescale) {
            factor = m_run == -INFINITY ? 0.f : ptx::ex2(m_run - m_new);
            m_run = m_new;
            l_run *= factor;
          }
          const float safe = m_run == -INFINITY ? 0.f : m_run;
          // P = exp2(s * scale * log2e - m) with packed f32x2 arithmetic; seven
          // element pairs in eight go through MUFU ex2 and the eighth through the
          // FMA-pipe polynomial (the split measured fastest at the C5 shape: the
          // polynomial costs about five times the issue slots of MUFU, and MUFU
          // alone would take as long as the tile's MMAs); pairs are packed with
          // cvt.rn (measured 1.4 % faster than integer rounding at that shape).
          uint32_t pk[kHN / 2];
          uint64_t sum2[2] = {ptx::f2pack(0.f, 0.f), ptx::f2pack(0.f, 0.f)};
          // Dropout (kDrop): keep bits of this half's 64 keys, from the counter-based
          // generator the generic kernels use (dropout.cuh); P.V sees p * keep / (1 - p),
          // the row sum l does not.
          uint32_t keep[2] = {0xffffffffu, 0xffffffffu};
          if constexpr (kDrop) {
            const uint32_t bh = (uint32_t)(b * p.q_heads + h);
            keep[0] = keep[1] = 0u;
    #pragma unroll
            for (int j8 = 0; j8 < kHN / 8; ++j8)
              keep[j8 >> 2] |= dropout_keep8(args.drop, bh, (uint32_t)qi, (uint32_t)(k0 / 8 + j8)) << (8 * (j8 & 3));
          }
          auto dropped = [&](float pv, int c) -> float {
            if constexpr (kDrop) return (keep[c >> 5] >> (c & 31)) & 1u ? pv * args.drop.inv_keep_f : 0.f;
            return pv;
          };
          if (!need_mask) {
            const uint64_t sc2 = ptx::f2pack(qk_scale, qk_scale), ng2 = ptx::f2pack(-safe, -safe);
    #pragma unroll
            for (int c = 0; c < kHN; c += 2) {
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
            for (int c = 0; c < kHN; c += 2) {
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
          // P(j) into TMEM over the first 32 columns of this half's S(j) (already in
          // registers); P(j).V(j) reads it from there, and S(j+2) only overwrites it
          // after that MMA (one issuing thread, executed in order).
          ptx::tmem_st32(t_row + C::kColS + (uint32_t)(g & 1) * kBN + half * kHN,
                         pk);
          ptx::tmem_wait_st();
          // This half's O accumulator may be rescaled once P(j-1).V(j-1) of the half completed.
          if (j >= 1 &&
              !__all_sync(0xffffffffu, wait_bar(&bars->o_done[half], (g - 1) & 1, args.fault, FAULT_FWD_O))) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          // The rescale decision is per row; the TMEM round trip is warp-collective,
          // so the whole warp takes it when any row needs it (factor 1 elsewhere).
          if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
            if (!rescale) factor = 1.f;
            uint32_t o[32];
    #pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              ptx::tmem_ld32(t_row + col_o + 32 * c, o);
              ptx::tmem_wait_ld();
    #pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
              ptx::tmem_st32(t_row + col_o + 32 * c, o);
            }
            ptx::tmem_wait_st();
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&bars->p_full[half]);

        }
        // Epilogue of this query tile: both O accumulators final (each thread reads both).
        const int g_last = gk + n_tiles - 1;
        if (ok)
          ok = __all_sync(0xffffffffu, wait_bar(&bars->o_done[0], g_last & 1, args.fault, FAULT_FWD_O) &&
                                           wait_bar(&bars->o_done[1], g_last & 1, args.fault, FAULT_FWD_O));
        ptx::tc_fence_after();
        // Exchange (m, l) with the other half of the row (the previous exchange was read by both).
        if (ok && iq >= 1)
          ok = __all_sync(0xffffffffu, wait_bar(&bars->red_free, (iq - 1) & 1, args.fault, FAULT_FWD_O));
        red[(half * 128 + row) * 2 + 0] = m_run;
        red[(half * 128 + row) * 2 + 1] = l_run;
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->epi);
        ok = __all_sync(0xffffffffu, ok && wait_bar(&bars->epi, iq & 1, args.fault, FAULT_FWD_O));
        const float m_oth = red[((1 - half) * 128 + row) * 2 + 0];
        const float l_oth = red[((1 - half) * 128 + row) * 2 + 1];
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->red_free);
        const float m_a = half == 0 ? m_run : m_oth, l_a = half == 0 ? l_run : l_oth;
        const float m_b = half == 0 ? m_oth : m_run, l_b = half == 0 ? l_oth : l_run;
        const float m_all = fmaxf(m_a, m_b);
        const float m_safe = m_all == -INFINITY ? 0.f : m_all;
        const float f_a = m_a == -INFINITY ? 0.f : ptx::ex2(m_a - m_safe);
        const float f_b = m_b == -INFINITY ? 0.f : ptx::ex2(m_b - m_safe);
        const float l_all = l_a * f_a + l_b * f_b;
        const bool live_row = qi < p.q_len;
        const float inv = l_all > 0.f ? 1.f / l_all : 0.f;
        const float w_a = f_a * inv, w_b = f_b * inv;
        using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
        T* orow = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
                  (int64_t)qi * p.o.stride[2];
        // This thread writes output channels [half * D/2, half * D/2 + D/2).
    #pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          const uint32_t col = (uint32_t)(half * (D / 2) + 32 * c);
          uint32_t ra[32], rb[32];
          if (n_tiles > 0 && ok) {
            ptx::tmem_ld32(t_row + C::kColO + col, ra);
            ptx::tmem_ld32(t_row + C::kColO + D + col, rb);
            ptx::tmem_wait_ld();
          } else {
    #pragma unroll
            for (int e = 0; e < 32; ++e) ra[e] = rb[e] = 0u;
          }
          if (live_row) {
            float f[32];
    #pragma unroll
            for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(ra[e]) * w_a + __uint_as_float(rb[e]) * w_b;
    #pragma unroll
            for (int e = 0; e < 32; e += 8) {
              uint4 v;
              if (kBF16) {
                v = make_uint4(ptx::pack_bf16(f[e], f[e + 1]), ptx::pack_bf16(f[e + 2], f[e + 3]),
                               ptx::pack_bf16(f[e + 4], f[e + 5]), ptx::pack_bf16(f[e + 6], f[e + 7]));
              } else {
                v = make_uint4(ptx::pack_f16(f[e], f[e + 1]), ptx::pack_f16(f[e + 2], f[e + 3]),
                               ptx::pack_f16(f[e + 4], f[e + 5]), ptx::pack_f16(f[e + 6], f[e + 7]));
              }
              *reinterpret_cast<uint4*>(orow + col + e) = v;
            }
          }
        }
        if (live_row && p.lse && half == 0)
          reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] + (int64_t)qi * p.lse_stride[2]] =
              l_all > 0.f ? (m_all + __log2f(l_all)) * kLn2 : -INFINITY;
        // O of this tile is read: the next query tile's first P.V may overwrite it.
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->o_free);
        gk += n_tiles;
        ++iq;
      }
    })
  }
#undef TS_FOR_EACH_QTILE

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
bool tc_fwd_supported(const ts_attn_params& p) {
  if (p.dtype != TS_BF16 && p.dtype != TS_F16) return false;
  if (p.head_dim != p.value_dim || (p.head_dim != 64 && p.head_dim != 128)) return false;
  if (p.mask_kind != TS_MASK_NONE) return false;
  if (!(p.scale > 0.0)) return false;  // the row max is taken on raw scores, then scaled
  if (!view_tma_ok(p.q) || !view_tma_ok(p.k) || !view_tma_ok(p.v)) return false;
  if (p.o.stride[3] != 1 || reinterpret_cast<uintptr_t>(p.o.data) % 16 || (p.o.stride[2] * 2) % 16 ||
      (p.o.stride[1] * 2) % 16 || (p.o.stride[0] * 2) % 16)
    return false;
  return encode_fn() != nullptr;
}

bool gqa_decode_view(const ts_attn_params& p, ts_attn_params* view) {
  if (p.q_len != 1 || p.mask_kind != TS_MASK_NONE || p.kv_heads <= 0 || p.q_heads % p.kv_heads) return false;
  const int rep = p.q_heads / p.kv_heads;
  if (rep < 2 || rep > 128) return false;
  // The one query must see every valid key (the rows of the view share its position).
  if (p.is_causal && !p.kv_lens && p.causal_offset + 1 < p.kv_len) return false;
  if ((int64_t)p.batch * p.kv_heads < kGqaViewMinPairs) return false;
  ts_attn_params v = p;
  v.q_heads = p.kv_heads;
  v.q_len = rep;
  v.q.stride[1] = p.q.stride[1] * rep;
  v.q.stride[2] = p.q.stride[1];
  v.o.stride[1] = p.o.stride[1] * rep;
  v.o.stride[2] = p.o.stride[1];
  v.lse_stride[1] = p.lse_stride[1] * rep;
  v.lse_stride[2] = p.lse_stride[1];
  v.is_causal = 0;
  v.causal_offset = 0;
  if (!tc_fwd_supported(v)) return false;
  *view = v;
  return true;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      n <= 0)
    n = 148;
  return n;
}

// The persistent schedule pays off where each CTA of the one-tile-per-CTA grid
// would carry few key tiles, so its set-up and epilogue show (measured at
// B=8, H=16, T=4096: 839 against 786 TFLOP/s), and loses where rows are long
// (T=32768: 862 against 952; a 4096-row chunk at causal offsets up to 28672
// keys, 4 GPUs: 96 against 70 ms per prefill): causal, rows of at most 4096
// keys (offset + query length), no per-row lengths (units of unequal length
// would unbalance the static schedule), and at least two units per SM.
static bool use_persistent(const TcFwdArgs& a, int sms) {
  return a.p.is_causal && !a.p.kv_lens && a.p.causal_offset + a.p.q_len <= 32 * kBN && a.n_units >= 2 * sms;
}

// Kernel choice for problems of two or more query tiles: the two-tile kernel
// (attn_fwd_pair.cu) by default; TS_FWD_KERNEL = "tile" or "persistent" in the
// environment selects one of this file's kernels instead (read at every call,
// for tests and measurements of all three).
enum class FwdKernel { kDefault, kPair, kTile, kPersistent };
static FwdKernel fwd_kernel_env() {
  const char* e = getenv("TS_FWD_KERNEL");
  if (!e) return FwdKernel::kDefault;
  if (!strcmp(e, "pair")) return FwdKernel::kPair;
  if (!strcmp(e, "tile")) return FwdKernel::kTile;
  if (!strcmp(e, "persistent")) return FwdKernel::kPersistent;
  return FwdKernel::kDefault;
}

template <int D, bool BF16>
static cudaError_t launch_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const TcFwdArgs& a, cudaStream_t st, bool persistent) {
  const int sms = sm_count();
  if (persistent) {
    auto pk = a.drop.p > 0.f ? tc_fwd_persistent_kernel<D, BF16, true> : tc_fwd_persistent_kernel<D, BF16, false>;
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(pk), Cfg<D>::kSmem);
    if (e != cudaSuccess) return e;
    pk<<<dim3((unsigned)sms), 384, Cfg<D>::kSmem, st>>>(mq, mk, mv, a);
    return cudaGetLastError();
  }
  auto kern = a.drop.p > 0.f ? tc_fwd_kernel<D, BF16, true> : tc_fwd_kernel<D, BF16, false>;
  cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(kern), Cfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.n_q_tiles, a.p.q_heads, a.p.batch);
  kern<<<grid, 384, Cfg<D>::kSmem, st>>>(mq, mk, mv, a);
  return cudaGetLastError();
}

cudaError_t tc_forward(const ts_attn_params& p, uint32_t* fault, cudaStream_t st, const DropoutArgs* drop) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, p.q, p.dtype, p.batch, p.q_heads, p.q_len, p.head_dim, 128) ||
      !make_map(&mk, p.k, p.dtype, p.batch, p.kv_heads, p.kv_len, p.head_dim, 128) ||
      !make_map(&mv, p.v, p.dtype, p.batch, p.kv_heads, p.kv_len, p.value_dim, 128))
    return cudaErrorInvalidValue;
  TcFwdArgs a;
  a.p = p;
  a.n_q_tiles = ceil_div(p.q_len, kBM);
  a.half_x = (a.n_q_tiles + 1) / 2;
  a.n_units = p.batch * p.q_heads * a.half_x;
  a.fault = fault;
  a.drop = drop ? *drop : DropoutArgs{};
  // Without dropout, two or more query tiles run on the two-tile kernel, which
  // measured faster than both kernels of this file: C5 shape (T=32768) 1189
  // against 1066 TFLOP/s, C3 (T=4096) 886 against 843 (persistent) and 790
  // (one tile).
  // A single query tile (short prefill chunks, the grouped-query decode view)
  // keeps the one-tile kernel.
  // With dropout the one-tile kernels stay the default: the counter-based
  // generator lengthens each warpgroup's softmax, which the two-tile kernel
  // pays in full on its softmax -> P.V -> S chain (C3, p = 0.1: 362 against
  // 422 TFLOP/s for the persistent one-tile kernel).
  const FwdKernel env = fwd_kernel_env();
  if (a.n_q_tiles >= 2 && (env == FwdKernel::kPair || (env == FwdKernel::kDefault && a.drop.p == 0.f)))
    return tc_forward_pair(p, mq, mk, mv, fault, st, drop);
  const bool persistent = env == FwdKernel::kPersistent || (env == FwdKernel::kDefault && use_persistent(a, sm_count()));
  const bool bf = p.dtype == TS_BF16;
  if (p.head_dim == 64)
    return bf ? launch_tc<64, true>(mq, mk, mv, a, st, persistent) : launch_tc<64, false>(mq, mk, mv, a, st, persistent);
  return bf ? launch_tc<128, true>(mq, mk, mv, a, st, persistent) : launch_tc<128, false>(mq, mk, mv, a, st, persistent);
}

}  // namespace tsa
