// torch operator over the C ABI for the per-step drafter call.
//
// suffixgpu_b200::local_draft wraps sg_local_draft (the fused local step of
// SuffixGPUDrafter.propose_with_update / propose, proposer.py:186-331) so
// that the eager Python call costs one dispatcher hop: the outputs are
// allocated here (one int32 buffer and views) and the launch goes to the
// current torch stream. The drafter's settings arrive as a small host
// tensor holding an sg_draft_params struct; the batch shape comes from
// token_ids. Errors raise (TORCH_CHECK) with the library's status string.
// The sampled ids (and valid counts) may be page-locked host tensors and
// the draft / num_valid outputs may be caller-provided tensors, on the
// device or in page-locked host memory: the kernel then reads and writes
// those host buffers directly, with no separate copies. Host inputs are
// taken to be written by the CPU (not by GPU work still in flight).
// suffixgpu_b200::vllm_prepare wraps sg_vllm_prepare, the per-step input
// preparation of vLLM's GPU n-gram proposer, for the vLLM adapter.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cuda_runtime_api.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/suffixgpu.h"

namespace {

template <typename T>
T* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? t->data_ptr<T>() : nullptr;
}

void check_status(const char* what, int st) {
  // numbers are formatted here, into a std::string, before TORCH_CHECK
  TORCH_CHECK(st == SG_OK, std::string(what) + " failed: " +
                               sg_status_string(st) + " (status " +
                               std::to_string(st) + ", cuda error " +
                               std::to_string(sg_last_cuda_error()) + ")");
}

void check_cuda(cudaError_t e) {
  TORCH_CHECK(e == cudaSuccess, std::string("CUDA error in the global step: ") +
                                    cudaGetErrorString(e));
}


// Address the kernel uses for `t`: its data pointer for a tensor on
// `dev`, the mapped device address for a page-locked host tensor. Anything
// else (pageable host memory, another device) is refused before a launch.
int32_t* kernel_ptr(const at::Tensor& t, const at::Device& dev,
                   const char* what) {
  if (t.is_cuda()) {
    TORCH_CHECK(t.device() == dev, what, " is on ", t.device(),
                " but token_ids is on ", dev);
    return t.data_ptr<int32_t>();
  }
  TORCH_CHECK(t.device().is_cpu(), what, " must be a CUDA tensor or a "
              "page-locked host tensor");
  void* d = nullptr;
  TORCH_CHECK(t.numel() == 0 ||
                  sg_mapped_host_ptr(t.data_ptr<int32_t>(), &d) == SG_OK,
              what, " is a host tensor in pageable memory; pass a "
              "page-locked one (tensor.pin_memory()) or a CUDA tensor");
  return static_cast<int32_t*>(d);
}

std::vector<at::Tensor> local_draft(const at::Tensor& num_tokens,
                                    const at::Tensor& token_ids,
                                    const c10::optional<at::Tensor>& sampled,
                                    const c10::optional<at::Tensor>& valid_count,
                                    const c10::optional<at::Tensor>& mask,
                                    const at::Tensor& params, int64_t limit,
                                    bool extras,
                                    const c10::optional<at::Tensor>& out_draft,
                                    const c10::optional<at::Tensor>& out_num_valid) {
  TORCH_CHECK(token_ids.is_cuda() && num_tokens.is_cuda(),
              "suffixgpu_b200 ops need CUDA tensors");
  TORCH_CHECK(token_ids.scalar_type() == at::kInt && token_ids.dim() == 2 &&
                  token_ids.stride(1) == 1,
              "token_ids must be an int32 [B, S] tensor with unit column stride");
  TORCH_CHECK(params.device().is_cpu() &&
                  params.nbytes() == sizeof(sg_draft_params),
              "params must hold one sg_draft_params struct");
  const c10::cuda::CUDAGuard guard(token_ids.device());
  const int64_t b = token_ids.size(0), s = token_ids.size(1);
  sg_draft_params p;
  std::memcpy(&p, params.data_ptr(), sizeof(p));
  p.batch = static_cast<int32_t>(b);
  p.seq_len = static_cast<int32_t>(s);
  p.row_stride = token_ids.stride(0);
  const int64_t k = p.k;
  at::Tensor n = num_tokens;
  if (n.scalar_type() != at::kInt || !n.is_contiguous())
    n = n.to(at::kInt).contiguous();
  sg_local_inputs in{};
  in.num_tokens = n.data_ptr<int32_t>();
  in.token_ids = token_ids.data_ptr<int32_t>();
  in.limit = limit;
  const int64_t n_i32 = b * (k + 2 + (extras ? 2 : 0));
  at::Tensor buf = at::empty({n_i32}, token_ids.options());
  int32_t* base = buf.data_ptr<int32_t>();
  sg_local_outputs out{};
  out.draft = base;
  out.num_valid = base + b * k;
  std::vector<at::Tensor> res;
  res.reserve(7);
  const at::Device dev = token_ids.device();
  if (out_draft.has_value()) {
    const at::Tensor& o = *out_draft;
    TORCH_CHECK(o.scalar_type() == at::kInt && o.dim() == 2 &&
                    o.size(0) == b && o.size(1) == k && o.is_contiguous(),
                "out draft must be a contiguous int32 [B, k] tensor");
    out.draft = kernel_ptr(o, dev, "out draft");
    res.push_back(o);
  } else {
    res.push_back(buf.narrow(0, 0, b * k).view({b, k}));
  }
  if (out_num_valid.has_value()) {
    const at::Tensor& o = *out_num_valid;
    TORCH_CHECK(o.scalar_type() == at::kInt && o.dim() == 1 &&
                    o.size(0) == b && o.is_contiguous(),
                "out num_valid must be a contiguous int32 [B] tensor");
    out.num_valid = kernel_ptr(o, dev, "out num_valid");
    res.push_back(o);
  } else {
    res.push_back(buf.narrow(0, b * k, b));
  }
  at::Tensor samp, vc, msk;
  if (sampled.has_value()) {
    samp = *sampled;
    if (samp.is_cuda()) {
      if (samp.scalar_type() != at::kInt || !samp.is_contiguous())
        samp = samp.to(at::kInt).contiguous();
    } else {
      // a host tensor is read in place: no conversion into pageable memory
      TORCH_CHECK(samp.scalar_type() == at::kInt && samp.is_contiguous(),
                  "a host sampled tensor must be contiguous int32");
    }
    TORCH_CHECK(samp.dim() == 2 && samp.size(0) == b,
                "sampled must be [B, T] with B = token_ids rows");
    in.sampled = kernel_ptr(samp, dev, "sampled");
    in.sampled_cols = static_cast<int32_t>(samp.size(1));
    if (valid_count.has_value()) {
      vc = *valid_count;
      if (vc.is_cuda()) {
        vc = vc.to(at::kInt).contiguous();
      } else {
        TORCH_CHECK(vc.scalar_type() == at::kInt && vc.is_contiguous(),
                    "a host valid_count tensor must be contiguous int32");
      }
      TORCH_CHECK(vc.numel() >= b, "valid_count has fewer than B entries");
      in.valid_count = kernel_ptr(vc, dev, "valid_count");
    }
    // page-locked host inputs are the CPU's writes: the kernel may read
    // them before the previous kernel on the stream has finished
    in.host_ids = !samp.is_cuda() && (!vc.defined() || !vc.is_cuda());
    out.new_counts = base + b * (k + 1);
    res.push_back(buf.narrow(0, b * (k + 1), b));
  } else {
    res.push_back(buf.narrow(0, 0, 0));  // no update: empty new_counts
    if (mask.has_value()) {
      msk = mask->to(at::kBool).contiguous();
      in.mask = reinterpret_cast<const uint8_t*>(msk.data_ptr<bool>());
    }
  }
  if (extras) {
    at::Tensor score = at::empty({b}, token_ids.options().dtype(at::kFloat));
    at::Tensor rmask = at::empty({b}, token_ids.options().dtype(at::kBool));
    out.best_len = base + b * (k + 2);
    out.best_occ = base + b * (k + 3);
    out.best_score = score.data_ptr<float>();
    out.row_mask = reinterpret_cast<uint8_t*>(rmask.data_ptr<bool>());
    res.push_back(score);
    res.push_back(buf.narrow(0, b * (k + 2), b));
    res.push_back(buf.narrow(0, b * (k + 3), b));
    res.push_back(rmask);
  }
  const int st = sg_local_draft(
      &p, &in, &out,
      reinterpret_cast<sg_stream_t>(
          c10::cuda::getCurrentCUDAStream(token_ids.device().index()).stream()));
  check_status("sg_local_draft", st);
  return res;
}

// vLLM's update_token_ids_ngram (ngram_proposer_gpu.py) in one launch:
// returns [next_token_ids [B] int32, valid_sampled_tokens_count [B] int32,
// valid_sampled_token_ids [B, T] int32], B = sampled.size(0).
std::vector<at::Tensor> vllm_prepare(const at::Tensor& sampled,
                                     const c10::optional<at::Tensor>& discard,
                                     const at::Tensor& token_ids,
                                     const at::Tensor& num_tokens,
                                     int64_t vocab_size) {
  TORCH_CHECK(sampled.is_cuda() && token_ids.is_cuda() && num_tokens.is_cuda(),
              "suffixgpu_b200 ops need CUDA tensors");
  TORCH_CHECK(sampled.scalar_type() == at::kInt && sampled.dim() == 2,
              "sampled must be an int32 [B, T] tensor");
  TORCH_CHECK(token_ids.scalar_type() == at::kInt && token_ids.dim() == 2 &&
                  token_ids.stride(1) == 1,
              "token_ids must be an int32 [B, S] tensor with unit column stride");
  const c10::cuda::CUDAGuard guard(token_ids.device());
  at::Tensor samp = sampled.stride(1) == 1 ? sampled : sampled.contiguous();
  const int64_t b = samp.size(0), t = samp.size(1);
  TORCH_CHECK(token_ids.size(0) >= b && num_tokens.numel() >= b,
              "token_ids / num_tokens have fewer rows than sampled");
  at::Tensor n = num_tokens;
  if (n.scalar_type() != at::kInt || !n.is_contiguous())
    n = n.to(at::kInt).contiguous();
  at::Tensor disc;
  const uint8_t* dptr = nullptr;
  if (discard.has_value()) {
    TORCH_CHECK(discard->numel() >= b, "discard has fewer rows than sampled");
    disc = discard->to(at::kBool).contiguous();
    dptr = reinterpret_cast<const uint8_t*>(disc.data_ptr<bool>());
  }
  at::Tensor buf = at::empty({b * (2 + t)}, token_ids.options());
  int32_t* base = buf.data_ptr<int32_t>();
  const int st = sg_vllm_prepare(
      samp.data_ptr<int32_t>(), t > 0 ? samp.stride(0) : 0,
      static_cast<int32_t>(b), static_cast<int32_t>(t), dptr,
      token_ids.data_ptr<int32_t>(), token_ids.stride(0),
      static_cast<int32_t>(token_ids.size(1)), n.data_ptr<int32_t>(),
      vocab_size, base, base + b, base + 2 * b,
      reinterpret_cast<sg_stream_t>(
          c10::cuda::getCurrentCUDAStream(token_ids.device().index()).stream()));
  check_status("sg_vllm_prepare", st);
  return {buf.narrow(0, 0, b), buf.narrow(0, b, b),
          buf.narrow(0, 2 * b, b * t).view({b, t})};
}

// ---- the global step's two halves (GlobalIndex.start_global_step /
// finish_global_step): the same C ABI calls, stream fork and join as the
// Python orchestration, in one dispatcher hop each. Streams and events
// arrive as raw handles (0 = everything on the current stream); the
// caller owns every buffer (found = sa_len, sa_start, sa_end, d_len,
// d_pos, d_cnt).

void global_start(const at::Tensor& counts, const at::Tensor& token_ids,
                  const c10::optional<at::Tensor>& sampled,
                  const c10::optional<at::Tensor>& valid_count,
                  const c10::optional<at::Tensor>& mask, int64_t limit,
                  const at::Tensor& sa, const at::Tensor& corpus,
                  int64_t capacity, const at::Tensor& delta,
                  int64_t delta_capacity, const at::Tensor& delta_len,
                  const at::Tensor& caps, const at::Tensor& tails,
                  const at::Tensor& tail_len, const at::Tensor& row_mask,
                  at::TensorList found, int64_t max_occ, int64_t s0,
                  int64_t s1, int64_t ev0, int64_t ev1) {
  TORCH_CHECK(token_ids.is_cuda() && token_ids.scalar_type() == at::kInt &&
                  token_ids.dim() == 2 && token_ids.stride(1) == 1,
              "token_ids must be an int32 CUDA [B, S] tensor");
  TORCH_CHECK(counts.scalar_type() == at::kInt && counts.is_contiguous(),
              "counts must be contiguous int32");
  TORCH_CHECK(found.size() == 6, "found must hold six tensors");
  const c10::cuda::CUDAGuard guard(token_ids.device());
  const int64_t b = token_ids.size(0), s = token_ids.size(1);
  const int32_t p = static_cast<int32_t>(tails.size(1));
  const int32_t cnum = static_cast<int32_t>(caps.numel());
  auto cur = reinterpret_cast<cudaStream_t>(
      c10::cuda::getCurrentCUDAStream(token_ids.device().index()).stream());
  cudaStream_t st_tails = cur, st_sa = cur, st_delta = cur;
  if (s0 != 0) {
    st_tails = st_sa = reinterpret_cast<cudaStream_t>(s0);
    st_delta = reinterpret_cast<cudaStream_t>(s1);
    check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev0), cur));
    check_cuda(cudaStreamWaitEvent(st_tails,
                                   reinterpret_cast<cudaEvent_t>(ev0), 0));
  }
  const int32_t* samp = ptr_or_null<int32_t>(sampled);
  const int32_t t_cols = sampled.has_value()
      ? static_cast<int32_t>(sampled->size(1)) : 0;
  const int32_t* vc = sampled.has_value() ? ptr_or_null<int32_t>(valid_count)
                                          : nullptr;
  const uint8_t* m8 = sampled.has_value() ? nullptr
                                          : ptr_or_null<uint8_t>(mask);
  check_status("sg_gather_tails_update", sg_gather_tails_update(
      token_ids.data_ptr<int32_t>(), token_ids.stride(0),
      static_cast<int32_t>(s), counts.data_ptr<int32_t>(), samp, t_cols, vc,
      limit, m8, static_cast<int32_t>(b), p, tails.data_ptr<int32_t>(),
      tail_len.data_ptr<int64_t>(), row_mask.data_ptr<uint8_t>(),
      reinterpret_cast<sg_stream_t>(st_tails)));
  if (s0 != 0) {  // the delta scan needs the tails
    check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev1), st_tails));
    check_cuda(cudaStreamWaitEvent(st_delta,
                                   reinterpret_cast<cudaEvent_t>(ev1), 0));
  }
  check_status("sg_suffix_match_backoff", sg_suffix_match_backoff(
      sa.data_ptr<int32_t>(), corpus.data_ptr<int32_t>(), capacity,
      tails.data_ptr<int32_t>(), static_cast<int32_t>(b), p,
      tail_len.data_ptr<int64_t>(), p, caps.data_ptr<int64_t>(), cnum,
      row_mask.data_ptr<uint8_t>(), found[0].data_ptr<int64_t>(),
      found[1].data_ptr<int64_t>(), found[2].data_ptr<int64_t>(),
      reinterpret_cast<sg_stream_t>(st_sa)));
  check_status("sg_delta_match_backoff", sg_delta_match_backoff(
      delta.data_ptr<int32_t>(), delta_capacity,
      delta_len.data_ptr<int64_t>(), tails.data_ptr<int32_t>(),
      static_cast<int32_t>(b), p, tail_len.data_ptr<int64_t>(), p,
      caps.data_ptr<int64_t>(), cnum, static_cast<int32_t>(max_occ),
      row_mask.data_ptr<uint8_t>(), found[3].data_ptr<int64_t>(),
      found[4].data_ptr<int64_t>(), found[5].data_ptr<int64_t>(),
      reinterpret_cast<sg_stream_t>(st_delta)));
}

// Returns SG_OK, or SG_ERR_UNSUPPORTED when the fused step does not fit
// shared memory (the caller then runs the separate steps).
int64_t global_finish(at::TensorList found, const at::Tensor& row_mask,
                      const at::Tensor& sa, const at::Tensor& corpus,
                      int64_t capacity, const at::Tensor& delta,
                      int64_t delta_capacity, const at::Tensor& delta_len,
                      int64_t max_occ, int64_t k, bool has_spec,
                      double spec_factor, double spec_offset,
                      double min_prob, double alpha,
                      const at::Tensor& local_score, const at::Tensor& draft,
                      const at::Tensor& num_valid, int64_t s0, int64_t s1,
                      int64_t ev2, int64_t ev3) {
  TORCH_CHECK(found.size() == 6, "found must hold six tensors");
  const c10::cuda::CUDAGuard guard(draft.device());
  auto cur = reinterpret_cast<cudaStream_t>(
      c10::cuda::getCurrentCUDAStream(draft.device().index()).stream());
  if (s0 != 0) {
    check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev2),
                               reinterpret_cast<cudaStream_t>(s0)));
    check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev3),
                               reinterpret_cast<cudaStream_t>(s1)));
    check_cuda(cudaStreamWaitEvent(cur, reinterpret_cast<cudaEvent_t>(ev2), 0));
    check_cuda(cudaStreamWaitEvent(cur, reinterpret_cast<cudaEvent_t>(ev3), 0));
  }
  const int32_t b = static_cast<int32_t>(row_mask.size(0));
  const int32_t cnum = static_cast<int32_t>(found[0].size(1));
  const int st = sg_global_draft(
      found[0].data_ptr<int64_t>(), found[1].data_ptr<int64_t>(),
      found[2].data_ptr<int64_t>(), found[3].data_ptr<int64_t>(),
      found[4].data_ptr<int64_t>(), found[5].data_ptr<int64_t>(),
      sa.data_ptr<int32_t>(), corpus.data_ptr<int32_t>(), capacity,
      delta.data_ptr<int32_t>(), delta_capacity,
      delta_len.data_ptr<int64_t>(), b, cnum, static_cast<int32_t>(max_occ),
      static_cast<int32_t>(k), has_spec ? 1 : 0,
      static_cast<float>(spec_factor), static_cast<float>(spec_offset),
      static_cast<float>(min_prob), static_cast<float>(alpha),
      local_score.data_ptr<float>(), row_mask.data_ptr<uint8_t>(),
      draft.data_ptr<int32_t>(), num_valid.data_ptr<int32_t>(),
      reinterpret_cast<sg_stream_t>(cur));
  if (st == SG_ERR_UNSUPPORTED) return st;
  check_status("sg_global_draft", st);
  return SG_OK;
}

}  // namespace

TORCH_LIBRARY(suffixgpu_b200, m) {
  m.def(
      "local_draft(Tensor num_tokens, Tensor token_ids, Tensor? sampled, "
      "Tensor? valid_count, Tensor? mask, Tensor params, int limit, "
      "bool extras, Tensor? out_draft=None, Tensor? out_num_valid=None) "
      "-> Tensor[]");
  m.def(
      "vllm_prepare(Tensor sampled, Tensor? discard, Tensor token_ids, "
      "Tensor num_tokens, int vocab_size) -> Tensor[]");
  m.def(
      "global_start(Tensor counts, Tensor token_ids, Tensor? sampled, "
      "Tensor? valid_count, Tensor? mask, int limit, Tensor sa, "
      "Tensor corpus, int capacity, Tensor delta, int delta_capacity, "
      "Tensor delta_len, Tensor caps, Tensor tails, Tensor tail_len, "
      "Tensor row_mask, Tensor[] found, int max_occ, int s0, int s1, "
      "int ev0, int ev1) -> ()");
  m.def(
      "global_finish(Tensor[] found, Tensor row_mask, Tensor sa, "
      "Tensor corpus, int capacity, Tensor delta, int delta_capacity, "
      "Tensor delta_len, int max_occ, int k, bool has_spec, "
      "float spec_factor, float spec_offset, float min_prob, float alpha, "
      "Tensor local_score, Tensor draft, Tensor num_valid, int s0, int s1, "
      "int ev2, int ev3) -> int");
}

TORCH_LIBRARY_IMPL(suffixgpu_b200, CUDA, m) {
  m.impl("local_draft", &local_draft);
  m.impl("vllm_prepare", &vllm_prepare);
  m.impl("global_start", &global_start);
  m.impl("global_finish", &global_finish);
}
