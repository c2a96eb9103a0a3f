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

#include <cstring>
#include <vector>

#include "../../include/suffixgpu.h"

namespace {

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
  TORCH_CHECK(st == SG_OK, "sg_local_draft failed: ", sg_status_string(st),
              " (status ", st, ", cuda error ", sg_last_cuda_error(), ")");
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
  TORCH_CHECK(st == SG_OK, "sg_vllm_prepare failed: ", sg_status_string(st),
              " (status ", st, ", cuda error ", sg_last_cuda_error(), ")");
  return {buf.narrow(0, 0, b), buf.narrow(0, b, b),
          buf.narrow(0, 2 * b, b * t).view({b, t})};
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
}

TORCH_LIBRARY_IMPL(suffixgpu_b200, CUDA, m) {
  m.impl("local_draft", &local_draft);
  m.impl("vllm_prepare", &vllm_prepare);
}
