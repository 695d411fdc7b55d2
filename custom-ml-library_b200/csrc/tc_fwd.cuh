// Entry points of the tcgen05 prefill forward (attn_fwd_tc.cu).
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "dropout.cuh"

namespace tsa {
// True when the tensor-core kernel takes this problem.
bool tc_fwd_supported(const ts_attn_params& p);
// `drop` set: attention dropout on P before P.V (the generic kernels' mask).
cudaError_t tc_forward(const ts_attn_params& p, uint32_t* fault, cudaStream_t stream,
                       const DropoutArgs* drop = nullptr);

// The two-query-tile kernel (attn_fwd_pair.cu) on the maps tc_forward built
// (128-row boxes of Q, K and V).
cudaError_t tc_forward_pair(const ts_attn_params& p, const CUtensorMap& mq, const CUtensorMap& mk,
                            const CUtensorMap& mv, uint32_t* fault, cudaStream_t stream, const DropoutArgs* drop);

// Fewest (batch, KV head) pairs for which a grouped-query decode step runs on
// the prefill kernel (one CTA per pair, no split along the keys): with fewer,
// the split-K decode keeps more SMs busy.
constexpr int64_t kGqaViewMinPairs = 64;

// A one-token decode step of a grouped-query problem (2 to 128 query heads per
// KV head, no explicit mask, the query seeing every valid key) as a prefill
// problem: the query heads of one KV head become the rows of one query tile,
// with no causal rule among them (same position) and the same key range and
// kv_lens.  The tcgen05 kernel then streams each KV head once with its whole
// group on the tensor cores.  Fills `view` and returns true when the problem
// qualifies, at least kGqaViewMinPairs pairs run and the tensor-core kernel
// takes the view.
bool gqa_decode_view(const ts_attn_params& p, ts_attn_params* view);
}  // namespace tsa
