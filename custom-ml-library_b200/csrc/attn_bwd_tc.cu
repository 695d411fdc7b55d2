// Attention backward on the tcgen05 tensor cores for bf16 / f16 inputs with
// D = Dv in {64, 128}.
//
// Replaces the blockwise VJP of tensorsmith's nn/attention.py:220-247: per
// (query block, key block) p = exp(S - LSE), dS = p * (dO.V^T - rowsum(dO*O))
// * scale, dQ += dS K, dK += dS^T Q, dV += p^T dO, with dK/dV summed over the
// query heads of a KV group (:245-247).
//
// One CTA = 128 keys of one (batch, KV head); it loops over 64-row query tiles
// of every query head of the group (causal: only tiles that see the keys).
// Per query tile five MMAs run with TMEM accumulators (lane = key for the
// first four, lane = channel for the last):
//   S^T  = K  Q^T     [128 x 64]   A = K   (smem, K-major)  B = Q   (K-major)
//   dP^T = V  dO^T    [128 x 64]   A = V   (smem, K-major)  B = dO  (K-major)
//   dV  += P^T dO     [128 x Dv]   A = P^T (TMEM)           B = dO  (MN-major)
//   dK  += dS^T Q     [128 x D]    A = dS^T(TMEM)           B = Q   (MN-major)
//   dQ^T = K^T dS^T   [D x 64]     A = K   (smem, MN-major) B = dS^T(smem, MN-major)
// Two "softmax" warpgroups (thread = key row) form P^T and dS^T from S^T, dP^T
// and the tile's row statistics, one over query columns [0, 32) of every
// tile and one over [32, 64), and write them as bf16/f16 pairs into TMEM
// (A operands of dV / dK) and dS^T also into a 128-byte-swizzled shared tile
// (B operand of dQ^T).  Row statistics (-LSE*log2e, -delta, padded to the
// 64-row tile) are written by a small preprocess kernel and copied by the
// producer beside each Q/dO tile (3-stage ring).  dQ^T is read by the epilogue
// warpgroup (thread = channel), staged channel-major in shared memory with
// 128-bit stores and added into a tile-major fp32 dQ accumulator with one bulk
// reduce-add (cp.reduce.async.bulk .add.f32) per query tile; a final kernel
// transposes and converts it.  dK/dV stay in TMEM for the whole CTA (no
// atomics, GQA summed).
//
// Warps: 0 TMA producer, 1 MMA issuer, 2 TMEM allocator, 4-7 and 12-15
// softmax (P^T, dS^T of their column half, then the dK resp. dV epilogue),
// 8-11 dQ epilogue.  No TMA load uses cluster multicast.
//
// Measured against the one-warpgroup softmax with row-major dQ staging (C3,
// bf16, D=128): splitting the columns over two warpgroups 531 -> 567 TFLOP/s,
// and channel-major staging with 128-bit stores (16 stores per thread instead
// of 64 scalar ones) 567 -> 659.  Double-buffering the staging (which needs a
// 2-stage Q/dO ring to fit in shared memory) and per-warp 4 KB reduces were
// slower at T = 32768.
#include <type_traits>

#include "ptx.cuh"
#include "simt.cuh"
#include "tc_bwd.cuh"
#include "tc_util.cuh"

namespace tsa {

namespace {

constexpr int kBN = 128;  // keys per CTA
constexpr int kBM = 64;   // query rows per iteration
constexpr int kQStages = 3;  // Q / dO / row-statistics ring depth
constexpr int kKSlab = 128 * 128;  // 128 rows x 128 B
constexpr int kQSlab = 64 * 128;   // 64 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;

template <int D> struct BwdCfg {
  static constexpr int kSlabs = D / 64;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kSlabs * kKSlab;
  static constexpr int kOffQ = kOffV + kSlabs * kKSlab;                // kQStages stages
  static constexpr int kOffDO = kOffQ + kQStages * kSlabs * kQSlab;     // kQStages stages
  static constexpr int kOffDS = kOffDO + kQStages * kSlabs * kQSlab;
  static constexpr int kOffStat = kOffDS + kKSlab;             // [stage][-LSE*log2e | -delta][64] floats
  static constexpr int kOffDQ = kOffStat + kQStages * 2 * kBM * 4;  // [D][64] fp32 dQ^T staging
  static constexpr int kDQTile = kBM * D * 4;
  static constexpr int kOffBar = kOffDQ + 1 * kDQTile;
  static constexpr int kUsed = kOffBar + 256 + 1024;
  // One CTA per SM: the kernel owns all 512 TMEM columns.
  static constexpr int kSmem = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
  static constexpr uint32_t kColDK = 0, kColDV = 128, kColS = 256, kColDP = 320, kColDQ = 384;
  // P^T and dS^T as bf16/f16 pairs (A operands of dV / dK read from TMEM).
  static constexpr uint32_t kColP = 448, kColDSt = 480;
};

struct BwdBars {
  uint64_t kv_full;
  uint64_t qdo_full[kQStages], qdo_empty[kQStages];
  uint64_t s_full, s_free, p_full, b_done, dq_free, drain;
  uint32_t tmem_base;
};

struct TcBwdArgs {
  ts_attn_params p;  // forward problem (q, k, v, o, lse)
  ts_view4 dk, dv;
  float* stats;      // [B*Hq][2][t_pad]: -LSE*log2e (-inf: no row / fully masked), -delta (0: no row)
  int t_pad;         // Tq rounded up to the 64-row query tile
  float* dq_acc;     // [B*Hq][t_pad / 64][D][64] fp32: per 64-row tile, channel d's 64 rows as
                     // 16-byte chunks, chunk j stored at index (j ^ (d & 7))
  int n_k_tiles;
  uint32_t* fault;
  DropoutArgs drop;  // used by the kDrop instantiation only
};

}  // namespace

template <int D, bool kBF16, bool kDrop>
__global__ void __launch_bounds__(512, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  TcBwdArgs args) {
  using C = BwdCfg<D>;
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  const ts_attn_params& p = args.p;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + C::kOffBar);
  unsigned char* sK = smem + C::kOffK;
  unsigned char* sV = smem + C::kOffV;
  unsigned char* sQ = smem + C::kOffQ;
  unsigned char* sDO = smem + C::kOffDO;
  unsigned char* sDS = smem + C::kOffDS;
  float* sStat = reinterpret_cast<float*>(smem + C::kOffStat);  // [buf][lse2 | delta][64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int rep = p.q_heads / p.kv_heads;
  const int k0 = kt * kBN;

  int kv_end = p.kv_len;
  int64_t offset = p.causal_offset;
  if (p.kv_lens) {
    kv_end = min(kv_end, max(0, p.kv_lens[b]));
    offset = (int64_t)kv_end - p.q_len;
  }
  const int n_qt_all = ceil_div(p.q_len, kBM);
  int qt_start = 0;
  if (p.is_causal) qt_start = (int)(i64max(0, (int64_t)k0 - offset) / kBM);
  const int n_qt = k0 < kv_end ? max(0, n_qt_all - qt_start) : 0;
  const int n_it = rep * n_qt;
  const bool dead = fault_set(args.fault);

  if (threadIdx.x == 0) {
    ptx::mbar_init(&bars->kv_full, 1);
    for (int s = 0; s < kQStages; ++s) {
      ptx::mbar_init(&bars->qdo_full[s], 1);
      ptx::mbar_init(&bars->qdo_empty[s], 1);
    }
    ptx::mbar_init(&bars->s_full, 1);
    ptx::mbar_init(&bars->s_free, 8);
    ptx::mbar_init(&bars->p_full, 8);
    ptx::mbar_init(&bars->b_done, 1);
    ptx::mbar_init(&bars->dq_free, 4);
    ptx::mbar_init(&bars->drain, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 2) {
    ptx::tmem_alloc(&bars->tmem_base, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  auto it_head = [&](int it) { return hk * rep + it / n_qt; };
  auto it_q0 = [&](int it) { return (qt_start + it % n_qt) * kBM; };

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0 && n_it > 0 && !dead) {
      ptx::prefetch_tensormap(&tm_q);
      ptx::prefetch_tensormap(&tm_k);
      ptx::prefetch_tensormap(&tm_v);
      ptx::prefetch_tensormap(&tm_do);
      ptx::mbar_expect_tx(&bars->kv_full, 2 * C::kSlabs * kKSlab);
      for (int sl = 0; sl < C::kSlabs; ++sl) {
        ptx::tma_load_4d(sK + sl * kKSlab, &tm_k, 64 * sl, k0, hk, b, &bars->kv_full);
        ptx::tma_load_4d(sV + sl * kKSlab, &tm_v, 64 * sl, k0, hk, b, &bars->kv_full);
      }
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % kQStages;
        if (it >= kQStages && !wait_bar(&bars->qdo_empty[s], ((it / kQStages) - 1) & 1, args.fault, FAULT_FWD_EMPTY))
          break;
        const int h = it_head(it), q0 = it_q0(it);
        ptx::mbar_expect_tx(&bars->qdo_full[s], 2 * C::kSlabs * kQSlab + 2 * kBM * 4);
        for (int sl = 0; sl < C::kSlabs; ++sl) {
          ptx::tma_load_4d(sQ + (s * C::kSlabs + sl) * kQSlab, &tm_q, 64 * sl, q0, h, b, &bars->qdo_full[s]);
          ptx::tma_load_4d(sDO + (s * C::kSlabs + sl) * kQSlab, &tm_do, 64 * sl, q0, h, b, &bars->qdo_full[s]);
        }
        // The tile's row statistics (padded rows: p = 0, delta = 0) ride on the same barrier.
        const float* st = args.stats + ((int64_t)b * p.q_heads + h) * 2 * args.t_pad + q0;
        ptx::bulk_g2s(sStat + s * 2 * kBM, st, kBM * 4, &bars->qdo_full[s]);
        ptx::bulk_g2s(sStat + s * 2 * kBM + kBM, st + args.t_pad, kBM * 4, &bars->qdo_full[s]);
        issued = it + 1;
      }
      (void)wait_bar(&bars->kv_full, 0, nullptr, FAULT_FWD_DRAIN);
      for (int it = max(0, issued - kQStages); it < issued; ++it)
        (void)wait_bar(&bars->qdo_full[it % kQStages], (it / kQStages) & 1, nullptr, FAULT_FWD_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0 && n_it > 0 && !dead) {
      constexpr uint32_t id_s = ptx::idesc_f16(kBF16, 128, kBM, false, false);
      constexpr uint32_t id_dkv = ptx::idesc_f16(kBF16, 128, D, false, true);
      constexpr uint32_t id_dq = ptx::idesc_f16(kBF16, 128, kBM, true, true);
      const uint32_t aK = ptx::smem_u32(sK), aV = ptx::smem_u32(sV), aQ = ptx::smem_u32(sQ),
                     aDO = ptx::smem_u32(sDO), aDS = ptx::smem_u32(sDS);
      bool ok = wait_bar(&bars->kv_full, 0, args.fault, FAULT_FWD_KV);
      auto issue_a = [&](int it) -> bool {
        const int s = it % kQStages;
        if (!wait_bar(&bars->qdo_full[s], (it / kQStages) & 1, args.fault, FAULT_FWD_KV)) return false;
        ptx::tc_fence_after();
        const uint32_t q = aQ + s * C::kSlabs * kQSlab, dO = aDO + s * C::kSlabs * kQSlab;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * kKSlab + (kk & 3) * 32, qo = (kk >> 2) * kQSlab + (kk & 3) * 32;
          ptx::mma_f16_ss(tmem + C::kColS, ptx::sw128_desc(aK + ko, 16, 1024), ptx::sw128_desc(q + qo, 16, 1024),
                          id_s, kk > 0 ? 1u : 0u);
          ptx::mma_f16_ss(tmem + C::kColDP, ptx::sw128_desc(aV + ko, 16, 1024),
                          ptx::sw128_desc(dO + qo, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&bars->s_full);
        return true;
      };
      if (ok) ok = issue_a(0);
      for (int it = 0; it < n_it && ok; ++it) {
        if (it + 1 < n_it) {
          if (!wait_bar(&bars->s_free, it & 1, args.fault, FAULT_FWD_S) || !issue_a(it + 1)) {
            ok = false;
            break;
          }
        }
        if (!wait_bar(&bars->p_full, it & 1, args.fault, FAULT_FWD_P) ||
            (it >= 1 && !wait_bar(&bars->dq_free, (it - 1) & 1, args.fault, FAULT_FWD_O))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const int s = it % kQStages;
        const uint32_t q = aQ + s * C::kSlabs * kQSlab, dO = aDO + s * C::kSlabs * kQSlab;
#pragma unroll
        for (int kk = 0; kk < kBM / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          ptx::mma_f16_ts(tmem + C::kColDV, tmem + C::kColP + kk * 8,
                          ptx::sw128_desc(dO + kk * 16 * 128, kQSlab, 1024), id_dkv, acc);
          ptx::mma_f16_ts(tmem + C::kColDK, tmem + C::kColDSt + kk * 8,
                          ptx::sw128_desc(q + kk * 16 * 128, kQSlab, 1024), id_dkv, acc);
        }
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          ptx::mma_f16_ss(tmem + C::kColDQ, ptx::sw128_desc(aK + kk * 16 * 128, kKSlab, 1024),
                          ptx::sw128_desc(aDS + kk * 16 * 128, kQSlab, 1024), id_dq, kk > 0 ? 1u : 0u);
        ptx::mma_commit(&bars->b_done);
        ptx::mma_commit(&bars->qdo_empty[s]);
      }
      ptx::mma_commit(&bars->drain);
      (void)wait_bar(&bars->drain, 0, nullptr, FAULT_FWD_DRAIN);
    }
  } else if ((warp >= 4 && warp < 8) || warp >= 12) {
    // ------------------- P^T / dS^T (thread = key row) ---------------------
    // Two warpgroups over the same 128 key rows: warps 4-7 take query columns
    // [0, 32) of every tile, warps 12-15 columns [32, 64).
    const int half = warp >= 12 ? 1 : 0;
    const int row = (warp & 3) * 32 + lane;
    const int key = k0 + row;
    const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float sl2 = (float)p.scale * kLog2e, scale = (float)p.scale;
    bool ok = !dead;
    // Every softmax warp runs all n_it iterations and reaches every named
    // barrier; after a failed wait it only skips the work (no early exit).
    for (int it = 0; it < n_it; ++it) {
      const int q0 = it_q0(it);
      const float* nlse2 = sStat + (it % kQStages) * 2 * kBM;
      const float* ndlt = nlse2 + kBM;
      // Warp-uniform outcomes: the tcgen05.ld below are warp-collective.  The
      // statistics landed with the Q/dO stage (already complete when S is).
      if (ok) ok = __all_sync(0xffffffffu, wait_bar(&bars->qdo_full[it % kQStages], (it / kQStages) & 1, args.fault, FAULT_FWD_KV) &&
                                               wait_bar(&bars->s_full, it & 1, args.fault, FAULT_FWD_S));
      if (ok) {
        ptx::tc_fence_after();
        const bool key_ok = key < kv_end;
        // Query columns this key row is visible to: col >= c_min (causal rule
        // i + offset >= key), none when the key is past the row's end.
        const int64_t cm = p.is_causal ? (int64_t)key - offset - q0 : 0;
        const int c_min = key_ok ? (int)i64max(0, i64min(kBM, cm)) : kBM;
        {
          uint32_t rs[32], rd[32];
          ptx::tmem_ld32(t_row + C::kColS + 32 * half, rs);
          ptx::tmem_ld32(t_row + C::kColDP + 32 * half, rd);
          ptx::tmem_wait_ld();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&bars->s_free);
          uint32_t pk[16], dk[16];
          // -LSE*log2e and -delta of this group's columns, read as packed pairs
          // (64-bit shared-memory broadcasts) inside the element loop.
          const uint64_t* nl2 = reinterpret_cast<const uint64_t*>(nlse2 + 32 * half);
          const uint64_t* nd2 = reinterpret_cast<const uint64_t*>(ndlt + 32 * half);
          // Dropout (kDrop): keep bit of (this key, column 32*half + c) in bit c.  The
          // generator gives the bits of 8 consecutive keys per call, so the 8 lanes
          // of a key octet each draw one column of every 8 and swap bytes.
          uint32_t kb = 0xffffffffu;
          if constexpr (kDrop) {
            kb = 0u;
            const uint32_t bh = (uint32_t)(b * p.q_heads + it_head(it));
            const uint32_t j8 = (uint32_t)key >> 3;
            const int oct = lane & ~7, sub = lane & 7;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint32_t byte = dropout_keep8(args.drop, bh, (uint32_t)(q0 + 32 * half + 8 * g + sub), j8);
#pragma unroll
              for (int t = 0; t < 8; ++t)
                kb |= ((__shfl_sync(0xffffffffu, byte, oct + t) >> sub) & 1u) << (8 * g + t);
            }
          }
          const float dinv = kDrop ? args.drop.inv_keep_f : 1.f;
          // Columns below c_min are masked; warp-uniform fast path when none of this half is.
          const bool all_vis = __all_sync(0xffffffffu, c_min <= 32 * half);
          const uint64_t sl2x2 = ptx::f2pack(sl2, sl2), scx2 = ptx::f2pack(scale, scale);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            // p = exp2(s * scale * log2e - LSE * log2e); dS = p * scale * (dP - delta), in f32 pairs.
            const uint64_t x2 = ptx::fma2(ptx::f2pack(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sl2x2,
                                          nl2[c / 2]);
            float x0, x1;
            ptx::f2unpack(x2, x0, x1);
            float p0 = ptx::ex2(x0), p1 = ptx::ex2(x1);
            if (!all_vis) {
              const int col = 32 * half + c;
              p0 = col >= c_min ? p0 : 0.f;
              p1 = col + 1 >= c_min ? p1 : 0.f;
            }
            const uint64_t p2 = ptx::f2pack(p0, p1);
            uint64_t t2;
            if constexpr (kDrop) {
              // dV uses p * keep / (1 - p_drop); dS = p * (dP * keep / (1 - p_drop) - delta) * scale.
              const float f0 = (kb >> c) & 1u ? dinv : 0.f, f1 = (kb >> (c + 1)) & 1u ? dinv : 0.f;
              t2 = ptx::fma2(ptx::f2pack(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])), ptx::f2pack(f0, f1),
                             nd2[c / 2]);
              p0 *= f0;
              p1 *= f1;
            } else {
              t2 = ptx::add2(ptx::f2pack(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])), nd2[c / 2]);
            }
            const uint64_t ds2 = ptx::fma2(ptx::fma2(p2, scx2, 0ull), t2, 0ull);
            float d0, d1;
            ptx::f2unpack(ds2, d0, d1);
            pk[c / 2] = kBF16 ? ptx::pack_bf16(p0, p1) : ptx::pack_f16(p0, p1);
            dk[c / 2] = kBF16 ? ptx::pack_bf16(d0, d1) : ptx::pack_f16(d0, d1);
          }
          // P^T / dS^T buffers are free once the previous iteration's dV/dK/dQ MMAs completed.
          if (it >= 1)
            ok = __all_sync(0xffffffffu, wait_bar(&bars->b_done, (it - 1) & 1, args.fault, FAULT_FWD_O));
          if (ok) {
            // P^T and dS^T into TMEM (A operands of dV += P^T dO, dK += dS^T Q);
            // dS^T also into the swizzled shared tile, the B operand of dQ^T.
            ptx::tmem_st16(t_row + C::kColP + 16 * half, pk);
            ptx::tmem_st16(t_row + C::kColDSt + 16 * half, dk);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int chunk = half * 4 + c;
              const int off = row * 128 + ((chunk ^ (row & 7)) << 4);
              *reinterpret_cast<uint4*>(sDS + off) =
                  make_uint4(dk[4 * c], dk[4 * c + 1], dk[4 * c + 2], dk[4 * c + 3]);
            }
          }
        }
        if (ok) {
          ptx::tmem_wait_st();
          ptx::fence_proxy_async_smem();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&bars->p_full);
        }
      }
    }
    // dK / dV epilogue: TMEM rows -> global.
    if (ok && n_it > 0)
      ok = __all_sync(0xffffffffu, wait_bar(&bars->b_done, (n_it - 1) & 1, args.fault, FAULT_FWD_O));
    ptx::tc_fence_after();
    // tcgen05.ld is warp-collective (.sync.aligned): every lane loads, and only
    // the global stores are predicated on the key being inside the tensor.
    const bool store_row = key < p.kv_len;
    {
      const int which = half;
      const ts_view4& dst = which == 0 ? args.dk : args.dv;
      T* out = reinterpret_cast<T*>(dst.data) + (int64_t)b * dst.stride[0] + (int64_t)hk * dst.stride[1] +
               (int64_t)key * dst.stride[2];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (ok && n_it > 0) {
          ptx::tmem_ld32(t_row + (which == 0 ? C::kColDK : C::kColDV) + 32 * c, r);
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = 0u;
        }
        if (store_row) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            const float* f = reinterpret_cast<const float*>(r + e);
            uint4 v;
            if (kBF16)
              v = make_uint4(ptx::pack_bf16(f[0], f[1]), ptx::pack_bf16(f[2], f[3]), ptx::pack_bf16(f[4], f[5]),
                             ptx::pack_bf16(f[6], f[7]));
            else
              v = make_uint4(ptx::pack_f16(f[0], f[1]), ptx::pack_f16(f[2], f[3]), ptx::pack_f16(f[4], f[5]),
                             ptx::pack_f16(f[6], f[7]));
            *reinterpret_cast<uint4*>(out + 32 * c + e) = v;
          }
        }
      }
    }
  } else if (warp >= 8 && warp < 12) {
    // ----------------------- dQ epilogue (thread = channel) ----------------
    // dQ^T (lane = channel) -> a channel-major [D][64] fp32 staging tile (the
    // accumulator's tile layout) -> one bulk reduce-add into the fp32 dQ
    // accumulator per iteration, issued by the group's first thread.  Every dQ warp runs all
    // n_it iterations and reaches both named barriers; after a failed wait it
    // only skips the work.
    const int d = (warp - 8) * 32 + lane;
    const bool leader = threadIdx.x == 256;
    const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    float* stage = reinterpret_cast<float*>(smem + C::kOffDQ);
    bool ok = !dead;
    for (int it = 0; it < n_it; ++it) {
      if (ok) ok = __all_sync(0xffffffffu, wait_bar(&bars->b_done, it & 1, args.fault, FAULT_FWD_O));
      uint32_t r0[32], r1[32];
      if (ok) {
        ptx::tc_fence_after();
        ptx::tmem_ld32(t_row + C::kColDQ, r0);
        ptx::tmem_ld32(t_row + C::kColDQ + 32, r1);
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->dq_free);
      }
      // The staging tile is free once the previous iteration's reduce has read it.
      if (leader) ptx::bulk_wait_read<0>();
      asm volatile("bar.sync 2, 128;" ::: "memory");
      float* st = stage;
      if (ok && d < D) {
        // Channel d's 64 rows as 16 chunks of 4; chunk j at (j ^ (d & 7)) so
        // the 8 threads of each 128-bit store phase hit distinct banks.
        float4* rowp = reinterpret_cast<float4*>(st + d * kBM);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          rowp[j ^ (d & 7)] = make_float4(__uint_as_float(r0[4 * j]), __uint_as_float(r0[4 * j + 1]),
                                          __uint_as_float(r0[4 * j + 2]), __uint_as_float(r0[4 * j + 3]));
#pragma unroll
        for (int j = 0; j < 8; ++j)
          rowp[(8 + j) ^ (d & 7)] = make_float4(__uint_as_float(r1[4 * j]), __uint_as_float(r1[4 * j + 1]),
                                                __uint_as_float(r1[4 * j + 2]), __uint_as_float(r1[4 * j + 3]));
      }
      ptx::fence_proxy_async_smem();
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (leader && ok) {
        const int h = it_head(it), qt = it_q0(it) / kBM;
        ptx::bulk_reduce_add_f32(args.dq_acc + (((int64_t)b * p.q_heads + h) * (args.t_pad / kBM) + qt) * (D * kBM),
                                 st, (uint32_t)(D * kBM * 4));
        ptx::bulk_commit();
      }
    }
    if (leader) ptx::bulk_wait_all();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

// dq[b,h,i,:] = dq_acc (fp32, one channel-major [D][64] tile per 64 rows) converted
// to the input dtype: one CTA per (tile, b*h) transposes its tile through
// shared memory so both the read and the write are coalesced.
template <typename T, int D>
__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ acc, ts_view4 dq, int heads,
                                                         int len, int n_tiles) {
  __shared__ float tile[kBM][D + 1];
  const int bh = blockIdx.x, t = blockIdx.y;
  const float4* src = reinterpret_cast<const float4*>(acc + ((int64_t)bh * n_tiles + t) * (D * kBM));
  for (int idx = threadIdx.x; idx < D * (kBM / 4); idx += blockDim.x) {
    const int d = idx / (kBM / 4), j = (idx % (kBM / 4)) ^ (d & 7);
    const float4 v = src[idx];
    tile[4 * j][d] = v.x;
    tile[4 * j + 1][d] = v.y;
    tile[4 * j + 2][d] = v.z;
    tile[4 * j + 3][d] = v.w;
  }
  __syncthreads();
  const int b = bh / heads, h = bh % heads;
  T* out = reinterpret_cast<T*>(dq.data) + (int64_t)b * dq.stride[0] + (int64_t)h * dq.stride[1];
  for (int idx = threadIdx.x; idx < kBM * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D, i = t * kBM + r;
    if (i < len) out[(int64_t)i * dq.stride[2] + (int64_t)d * dq.stride[3]] = Elem<T>::from_acc(tile[r][d]);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static bool out_rows_ok(const ts_view4& v) {
  return v.stride[3] == 1 && reinterpret_cast<uintptr_t>(v.data) % 16 == 0 && (v.stride[2] * 2) % 16 == 0 &&
         (v.stride[1] * 2) % 16 == 0 && (v.stride[0] * 2) % 16 == 0;
}

bool tc_bwd_supported(const ts_attn_bwd_params& bp) {
  const ts_attn_params& p = bp.fwd;
  if (p.dtype != TS_BF16 && p.dtype != TS_F16) return false;
  if (p.head_dim != p.value_dim || (p.head_dim != 64 && p.head_dim != 128)) return false;
  if (p.mask_kind != TS_MASK_NONE || !p.lse) return false;
  if (!view_tma_ok(p.q) || !view_tma_ok(p.k) || !view_tma_ok(p.v) || !view_tma_ok(bp.dout)) return false;
  if (!out_rows_ok(bp.dk) || !out_rows_ok(bp.dv)) return false;
  return encode_fn() != nullptr;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static int t_padded(int q_len) { return ceil_div(q_len, kBM) * kBM; }

size_t tc_bwd_workspace(const ts_attn_bwd_params& bp) {
  const ts_attn_params& p = bp.fwd;
  const size_t rows = (size_t)p.batch * p.q_heads * t_padded(p.q_len);
  const size_t stats = (size_t)p.batch * p.q_heads * 2 * t_padded(p.q_len);
  return align256(stats * sizeof(float)) + align256(rows * p.head_dim * sizeof(float));
}

// stats[bh][0][i] = -LSE*log2e (-inf for a fully masked row or i >= Tq) and
// stats[bh][1][i] = -sum_c dO*O (0 for i >= Tq): the backward's row statistics
// (nn/attention.py:231), one warp per padded row.
template <typename T>
__global__ void bwd_stats_kernel(ts_attn_bwd_params bp, float* stats, int t_pad) {
  const ts_attn_params& p = bp.fwd;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)p.batch * p.q_heads * t_pad;
  if (warp >= total) return;
  const int i = (int)(warp % t_pad);
  const int64_t bh = warp / t_pad;
  const int h = (int)(bh % p.q_heads), b = (int)(bh / p.q_heads);
  float acc = 0.f;
  if (i < p.q_len) {
    const T* g = reinterpret_cast<const T*>(bp.dout.data) + b * bp.dout.stride[0] + h * bp.dout.stride[1] +
                 i * bp.dout.stride[2];
    const T* o = reinterpret_cast<const T*>(p.o.data) + b * p.o.stride[0] + h * p.o.stride[1] + i * p.o.stride[2];
    for (int c = lane; c < p.value_dim; c += 32)
      acc += Elem<T>::to_acc(g[c * bp.dout.stride[3]]) * Elem<T>::to_acc(o[c * p.o.stride[3]]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    float nl = -INFINITY;
    if (i < p.q_len) {
      const float l = reinterpret_cast<const float*>(p.lse)[(int64_t)b * p.lse_stride[0] +
                                                            (int64_t)h * p.lse_stride[1] + (int64_t)i * p.lse_stride[2]];
      nl = l == -INFINITY ? -INFINITY : -l * kLog2e;
    }
    stats[bh * 2 * t_pad + i] = nl;
    stats[bh * 2 * t_pad + t_pad + i] = i < p.q_len ? -acc : 0.f;
  }
}

template <int D, bool BF16>
static cudaError_t launch_bwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                              const CUtensorMap& mdo, const TcBwdArgs& a, cudaStream_t st) {
  auto kern = a.drop.p > 0.f ? tc_bwd_kernel<D, BF16, true> : tc_bwd_kernel<D, BF16, false>;
  cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(kern), BwdCfg<D>::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.n_k_tiles, a.p.kv_heads, a.p.batch);
  kern<<<grid, 512, BwdCfg<D>::kSmem, st>>>(mq, mk, mv, mdo, a);
  return cudaGetLastError();
}

cudaError_t tc_backward(const ts_attn_bwd_params& bp, void* ws, size_t ws_bytes, uint32_t* fault,
                        cudaStream_t st, const DropoutArgs* drop) {
  const ts_attn_params& p = bp.fwd;
  if (ws_bytes < tc_bwd_workspace(bp)) return cudaErrorInvalidValue;
  const int t_pad = t_padded(p.q_len);
  const size_t rows = (size_t)p.batch * p.q_heads * t_pad;
  const size_t n_stats = (size_t)p.batch * p.q_heads * 2 * t_pad;
  float* stats = reinterpret_cast<float*>(ws);
  float* dq_acc = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(ws) + align256(n_stats * sizeof(float)));
  CUtensorMap mq, mk, mv, mdo;
  if (!make_map(&mq, p.q, p.dtype, p.batch, p.q_heads, p.q_len, p.head_dim, kBM) ||
      !make_map(&mk, p.k, p.dtype, p.batch, p.kv_heads, p.kv_len, p.head_dim, kBN) ||
      !make_map(&mv, p.v, p.dtype, p.batch, p.kv_heads, p.kv_len, p.value_dim, kBN) ||
      !make_map(&mdo, bp.dout, p.dtype, p.batch, p.q_heads, p.q_len, p.value_dim, kBM))
    return cudaErrorInvalidValue;
  {
    const int64_t warps = (int64_t)p.batch * p.q_heads * t_pad;
    const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
    if (p.dtype == TS_BF16)
      bwd_stats_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(bp, stats, t_pad);
    else
      bwd_stats_kernel<__half><<<blocks, 256, 0, st>>>(bp, stats, t_pad);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(dq_acc, 0, rows * p.head_dim * sizeof(float), st);
  if (e != cudaSuccess) return e;
  TcBwdArgs a;
  a.p = p;
  a.dk = bp.dk;
  a.dv = bp.dv;
  a.stats = stats;
  a.t_pad = t_pad;
  a.dq_acc = dq_acc;
  a.n_k_tiles = ceil_div(p.kv_len, kBN);
  a.fault = fault;
  a.drop = drop ? *drop : DropoutArgs{};
  const bool bf = p.dtype == TS_BF16;
  if (p.head_dim == 64)
    e = bf ? launch_bwd<64, true>(mq, mk, mv, mdo, a, st) : launch_bwd<64, false>(mq, mk, mv, mdo, a, st);
  else
    e = bf ? launch_bwd<128, true>(mq, mk, mv, mdo, a, st) : launch_bwd<128, false>(mq, mk, mv, mdo, a, st);
  if (e != cudaSuccess) return e;
  const dim3 cgrid((unsigned)(p.batch * p.q_heads), (unsigned)(t_pad / kBM));
  const int n_tiles = t_pad / kBM;
  if (p.head_dim == 64) {
    if (bf)
      dq_convert_kernel<__nv_bfloat16, 64><<<cgrid, 256, 0, st>>>(dq_acc, bp.dq, p.q_heads, p.q_len, n_tiles);
    else
      dq_convert_kernel<__half, 64><<<cgrid, 256, 0, st>>>(dq_acc, bp.dq, p.q_heads, p.q_len, n_tiles);
  } else {
    if (bf)
      dq_convert_kernel<__nv_bfloat16, 128><<<cgrid, 256, 0, st>>>(dq_acc, bp.dq, p.q_heads, p.q_len, n_tiles);
    else
      dq_convert_kernel<__half, 128><<<cgrid, 256, 0, st>>>(dq_acc, bp.dq, p.q_heads, p.q_len, n_tiles);
  }
  return cudaGetLastError();
}

}  // namespace tsa
