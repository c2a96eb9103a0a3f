// vLLM glue: the per-step input preparation of vLLM's GPU n-gram proposer
// (vllm/v1/spec_decode/ngram_proposer_gpu.py, update_token_ids_ngram),
// which the V1 model runner calls before every ngram_gpu propose. vLLM
// computes it with about fifteen small torch ops; here it is one launch,
// one thread per request row:
//   valid[b, :]  = sampled[b, :], or all -1 when discard[b]
//   count[b]     = #{j : valid[b, j] != -1 and valid[b, j] < vocab_size}
//   next[b]      = valid[b, count[b] - 1] if count[b] > 0, else the row's
//                  last committed token token_ids[b, max(n[b] - 1, 0)]
// (the last valid token is read at index count - 1, as vLLM does, which
// assumes the accepted tokens are left-aligned). vLLM's gather faults for
// n[b] - 1 >= the row length; here that index is clamped to the row.
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

__global__ void vllm_prepare_kernel(const int32_t* __restrict__ sampled,
                                    int64_t sampled_stride, int32_t batch,
                                    int32_t cols,
                                    const uint8_t* __restrict__ discard,
                                    const int32_t* __restrict__ token_ids,
                                    int64_t row_stride, int32_t seq_len,
                                    const int32_t* __restrict__ num_tokens,
                                    int64_t vocab_size,
                                    int32_t* __restrict__ next_ids,
                                    int32_t* __restrict__ valid_count,
                                    int32_t* __restrict__ valid_sampled) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const bool drop = discard != nullptr && discard[b] != 0;
  const int32_t* srow = sampled + static_cast<int64_t>(b) * sampled_stride;
  int32_t* vrow = valid_sampled + static_cast<int64_t>(b) * cols;
  int c = 0;
  for (int j = 0; j < cols; ++j) {
    const int32_t v = drop ? -1 : srow[j];
    vrow[j] = v;
    c += (v != -1 && static_cast<int64_t>(v) < vocab_size) ? 1 : 0;
  }
  valid_count[b] = c;
  int32_t nx;
  if (c > 0) {
    nx = srow[c - 1];  // c > 0 implies the row is not discarded
  } else {
    int64_t i = static_cast<int64_t>(num_tokens[b]) - 1;
    if (i < 0) i = 0;
    if (i > seq_len - 1) i = seq_len - 1;
    nx = token_ids[static_cast<int64_t>(b) * row_stride + i];
  }
  next_ids[b] = nx;
}

}  // namespace sg

using namespace sg;

extern "C" int sg_vllm_prepare(const int32_t* sampled, int64_t sampled_stride,
                               int32_t batch, int32_t cols,
                               const uint8_t* discard,
                               const int32_t* token_ids, int64_t row_stride,
                               int32_t seq_len, const int32_t* num_tokens,
                               int64_t vocab_size, int32_t* next_ids,
                               int32_t* valid_count, int32_t* valid_sampled,
                               sg_stream_t stream) {
  if (batch < 0 || cols < 0 || seq_len < 0) return SG_ERR_INVALID;
  if (batch == 0) return SG_OK;
  if (cols > 0 && (!sampled || sampled_stride < cols || !valid_sampled))
    return SG_ERR_INVALID;
  if (!token_ids || seq_len < 1 || row_stride < seq_len || !num_tokens ||
      !next_ids || !valid_count)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  vllm_prepare_kernel<<<static_cast<unsigned>((batch + 127) / 128), 128, 0,
                        st>>>(sampled, sampled_stride, batch, cols, discard,
                              token_ids, row_stride, seq_len, num_tokens,
                              vocab_size, next_ids, valid_count,
                              valid_sampled);
  return check_launch();
}
