// Attention dropout (tensorsmith nn/attention.py:140-144 forward, :212-216
// backward): probabilities are multiplied by keep / (1 - p), keep = (u >= p)
// with u uniform in [0, 1) drawn per (batch, query head, query row, key).
//
// u comes from a counter-based generator, so the backward regenerates the
// forward's mask instead of storing it: Philox4x32 with 10 rounds (Salmon,
// Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011;
// round multipliers and Weyl key increments as published there).  Element
// (bh, i, j) of call `offset` uses counter {j / 8, i, bh, offset_lo}, key
// {seed_lo, seed_hi ^ offset_hi}, output word (j % 8) / 2 and its low (j even)
// or high (j odd) 16 bits w16; u = w16 * 2^-16, so keep = (w16 >= ceil(p * 2^16))
// and the keep probability is 1 - p within 2^-16.  One call covers 8 keys: the
// generator, not the softmax, bounds the dropout kernels' issue rate.
#pragma once
#include "common.cuh"

namespace tsa {

struct DropoutArgs {
  float p;          // drop probability, 0 <= p < 1
  uint32_t keep_min; // ceil(p * 2^16): a key is kept when its 16-bit uniform is >= this
  float inv_keep_f;  // 1 / (1 - p) as the reference scales in fp32: 1.0f / float(1 - p)
  double inv_keep_d; // the same in fp64
  uint64_t seed;
  uint64_t offset;
};

__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
  constexpr uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
  constexpr uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t hi0 = __umulhi(kMul0, ctr.x), lo0 = kMul0 * ctr.x;
    const uint32_t hi1 = __umulhi(kMul1, ctr.z), lo1 = kMul1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += kWeyl0;
    key.y += kWeyl1;
  }
  return ctr;
}

// Keep bits of keys j8*8 .. j8*8+7 of row (bh, i), in bits 0..7.
__device__ __forceinline__ uint32_t dropout_keep8(const DropoutArgs& d, uint32_t bh, uint32_t i, uint32_t j8) {
  const uint4 r = philox4x32_10(make_uint4(j8, i, bh, (uint32_t)d.offset),
                                make_uint2((uint32_t)d.seed, (uint32_t)(d.seed >> 32) ^ (uint32_t)(d.offset >> 32)));
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
  uint32_t bits = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    bits |= ((w[k] & 0xffffu) >= d.keep_min ? 1u : 0u) << (2 * k) | ((w[k] >> 16) >= d.keep_min ? 2u : 0u) << (2 * k);
  return bits;
}

__device__ __forceinline__ bool dropout_keep(const DropoutArgs& d, uint32_t bh, uint32_t i, uint32_t j) {
  return (dropout_keep8(d, bh, i, j >> 3) >> (j & 7)) & 1u;
}

template <typename A> __device__ __forceinline__ A dropout_scale(const DropoutArgs& d);
template <> __device__ __forceinline__ float dropout_scale<float>(const DropoutArgs& d) { return d.inv_keep_f; }
template <> __device__ __forceinline__ double dropout_scale<double>(const DropoutArgs& d) { return d.inv_keep_d; }

// Keep mask [B, Hq, Tq, Tk] as uint8 0/1 (tests, and callers that must see it).
cudaError_t dropout_mask(const DropoutArgs& d, int batch, int heads, int q_len, int kv_len, uint8_t* mask,
                         cudaStream_t stream);

}  // namespace tsa
