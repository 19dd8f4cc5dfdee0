// q3s_torch_ops.cpp -- torch.ops.q3s.*: the sampler as PyTorch operators.
//
// The reference's sampler is a sub-graph of its fused decode graph
// (scripts/export/talker_unified_modules.py:407-422 for codebook 0,
// scripts/export/utils.py:1178-1193 for one code-predictor stage, the loop of
// scripts/export/utils.py:1218-1237 for a frame).  These operators give
// torch-side callers (the export / validation code, an eager or traced
// decode step) the same call shapes, with schemas and Meta kernels so they
// trace, and CUDA kernels that fill a q3s_sample_desc / q3s_cp_frame_desc and
// call the C ABI of libq3s_sampler.so on the current CUDA stream.  Nothing is
// computed on the host; a bad argument raises (TORCH_CHECK), as the
// reference's executor raises on bad inputs (engine/backend/executor.py:
// 355-365).
//
//   sample_codebook0(logits, token_counts, gumbel_noise, temperature, penalty,
//                    suppress_mask=None, topk=50) -> (codec_token_0, updated_token_counts)
//   sample_codebook0_(logits, token_counts!, ...) -> codec_token_0   (counts + 1 in place)
//   sample_codebook0_packed(logits, history, offsets, uniforms, temperature, top_k, top_p,
//                           penalty, min_new_tokens, suppress_mask=None, eos_id=2150) -> ids
//   sample_cp_stage(logits, temperature=None, gumbel_noise=None, topk=50) -> ids
//   sample_cp_frame(logits[S,B,V], temperature, cp_gumbel_noise=None, topk=50) -> ids[B,S]
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstring>
#include <tuple>
#include <vector>

#include "q3s_sampler.h"

namespace {

using at::Tensor;

void check_status(q3s_status s, const char* what) {
  TORCH_CHECK(s == Q3S_OK, what, " failed (status ", static_cast<int>(s), "): ", q3s_last_error_string());
}

// [B,V] rows of the logits: [B,V] as is, [B,S,V] / [B,1,V] the last position
// (logits[:, -1, :], a strided view, no copy).
Tensor rows_2d(const Tensor& logits) {
  TORCH_CHECK(logits.is_cuda(), "q3s: logits must be a CUDA tensor (there is no CPU fallback)");
  TORCH_CHECK(logits.dim() == 2 || logits.dim() == 3, "q3s: logits must be [B,V] or [B,S,V], got ",
              logits.sizes());
  Tensor x = logits.dim() == 3 ? logits.select(1, logits.size(1) - 1) : logits;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat,
              "q3s: logits must be bf16 or fp32, got ", x.scalar_type());
  if (x.stride(1) != 1 || (x.size(0) > 1 && x.stride(0) < x.size(1))) x = x.contiguous();
  return x;
}

int32_t dtype_code(const Tensor& x) { return x.scalar_type() == at::kBFloat16 ? Q3S_DTYPE_BF16 : Q3S_DTYPE_F32; }

void same_device(const Tensor& t, const Tensor& ref, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.device() == ref.device(), "q3s: ", name, " must be on ", ref.device());
}

// A per-row parameter of B values ([B], [B,1]) or one value broadcast to the
// rows, as a contiguous tensor of `dt` kept alive in `keep`.
const void* row_param(const Tensor& t, int64_t B, at::ScalarType dt, const Tensor& ref, const char* name,
                      std::vector<Tensor>& keep) {
  same_device(t, ref, name);
  Tensor x = t.reshape({-1});
  TORCH_CHECK(x.numel() == B || x.numel() == 1, "q3s: ", name, " has ", x.numel(), " values for ", B, " rows");
  if (x.numel() != B) x = x.expand({B});
  x = x.to(dt).contiguous();
  keep.push_back(x);
  return x.data_ptr();
}

q3s_sample_desc base_desc(const Tensor& x, int32_t mode) {
  q3s_sample_desc d;
  std::memset(&d, 0, sizeof(d));
  d.struct_size = sizeof(q3s_sample_desc);
  d.mode = mode;
  d.batch = static_cast<int32_t>(x.size(0));
  d.vocab = static_cast<int32_t>(x.size(1));
  d.logits_dtype = dtype_code(x);
  d.logits_row_stride = x.size(0) > 1 ? x.stride(0) : x.size(1);
  d.logits = x.data_ptr();
  d.temperature_default = 1.0f;
  d.top_p_default = 1.0f;
  d.penalty_default = 1.0f;
  d.eos_id = -1;
  return d;
}

void launch(const q3s_sample_desc& d, const Tensor& ref) {
  check_status(q3s_sample(&d, c10::cuda::getCurrentCUDAStream(ref.get_device()).stream()), "q3s_sample");
}

// gumbel-mode inputs of the fused graph's codebook-0 sampler into `d`
void codebook0_inputs(q3s_sample_desc& d, const Tensor& x, const Tensor& token_counts, const Tensor& gumbel_noise,
                      const Tensor& temperature, const Tensor& penalty, const c10::optional<Tensor>& suppress,
                      int64_t topk, std::vector<Tensor>& keep) {
  const int64_t B = x.size(0), V = x.size(1);
  same_device(token_counts, x, "token_counts");
  TORCH_CHECK(token_counts.scalar_type() == at::kLong && token_counts.dim() == 2 && token_counts.size(0) == B &&
                  token_counts.size(1) == V && token_counts.stride(1) == 1,
              "q3s: token_counts must be int64 [B,V] with unit column stride");
  d.topk = static_cast<int32_t>(std::min<int64_t>(topk, V));
  d.token_counts = token_counts.data_ptr<int64_t>();
  d.token_counts_row_stride = B > 1 ? token_counts.stride(0) : V;
  same_device(gumbel_noise, x, "gumbel_noise");
  Tensor g = gumbel_noise.reshape({B, -1});
  if (g.scalar_type() != at::kFloat || g.stride(1) != 1) g = g.to(at::kFloat).contiguous();
  TORCH_CHECK(g.size(1) >= d.topk, "q3s: gumbel_noise has ", g.size(1), " columns, need ", d.topk);
  keep.push_back(g);
  d.gumbel_noise = g.data_ptr<float>();
  d.gumbel_row_stride = B > 1 ? g.stride(0) : g.size(1);
  d.temperature = static_cast<const float*>(row_param(temperature, B, at::kFloat, x, "temperature", keep));
  d.penalty = static_cast<const float*>(row_param(penalty, B, at::kFloat, x, "penalty", keep));
  if (suppress.has_value()) {
    same_device(*suppress, x, "suppress_mask");
    Tensor m = suppress->reshape({-1}).to(at::kBool).contiguous();
    TORCH_CHECK(m.numel() == V, "q3s: suppress_mask has ", m.numel(), " entries for vocab ", V);
    keep.push_back(m);
    d.suppress_mask = reinterpret_cast<const uint8_t*>(m.data_ptr<bool>());
  }
}

std::tuple<Tensor, Tensor> sample_codebook0(const Tensor& logits, const Tensor& token_counts,
                                            const Tensor& gumbel_noise, const Tensor& temperature,
                                            const Tensor& penalty, const c10::optional<Tensor>& suppress_mask,
                                            int64_t topk) {
  const Tensor x = rows_2d(logits);
  c10::cuda::CUDAGuard guard(x.device());
  std::vector<Tensor> keep;
  q3s_sample_desc d = base_desc(x, Q3S_DRAW_GUMBEL);
  codebook0_inputs(d, x, token_counts, gumbel_noise, temperature, penalty, suppress_mask, topk, keep);
  Tensor ids = at::empty({x.size(0)}, x.options().dtype(at::kLong));
  Tensor counts = at::empty({x.size(0), x.size(1)}, token_counts.options());
  d.ids_i64 = ids.data_ptr<int64_t>();
  d.counts_out = counts.data_ptr<int64_t>();
  d.counts_out_row_stride = x.size(1);
  launch(d, x);
  return {ids, counts};
}

Tensor sample_codebook0_(const Tensor& logits, Tensor& token_counts, const Tensor& gumbel_noise,
                         const Tensor& temperature, const Tensor& penalty, const c10::optional<Tensor>& suppress_mask,
                         int64_t topk) {
  const Tensor x = rows_2d(logits);
  c10::cuda::CUDAGuard guard(x.device());
  std::vector<Tensor> keep;
  q3s_sample_desc d = base_desc(x, Q3S_DRAW_GUMBEL);
  codebook0_inputs(d, x, token_counts, gumbel_noise, temperature, penalty, suppress_mask, topk, keep);
  Tensor ids = at::empty({x.size(0)}, x.options().dtype(at::kLong));
  d.ids_i64 = ids.data_ptr<int64_t>();
  d.counts_out = token_counts.data_ptr<int64_t>();  // the row's one count + 1, in place
  d.counts_out_row_stride = d.token_counts_row_stride;
  launch(d, x);
  return ids;
}

Tensor sample_codebook0_packed(const Tensor& logits, const Tensor& history, const Tensor& offsets,
                               const Tensor& uniforms, const Tensor& temperature, const Tensor& top_k,
                               const Tensor& top_p, const Tensor& penalty, const Tensor& min_new_tokens,
                               const c10::optional<Tensor>& suppress_mask, int64_t eos_id) {
  const Tensor x = rows_2d(logits);
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.size(0), V = x.size(1);
  std::vector<Tensor> keep;
  q3s_sample_desc d = base_desc(x, Q3S_DRAW_ICDF);
  same_device(history, x, "history");
  same_device(offsets, x, "offsets");
  Tensor h = history.reshape({-1}).to(at::kInt).contiguous();
  Tensor o = offsets.reshape({-1}).to(at::kInt).contiguous();
  TORCH_CHECK(o.numel() == B + 1, "q3s: offsets has ", o.numel(), " entries for ", B, " rows (need B+1)");
  keep.push_back(h);
  keep.push_back(o);
  d.history = h.numel() ? h.data_ptr<int32_t>() : o.data_ptr<int32_t>();
  d.offsets = o.data_ptr<int32_t>();
  d.history_len = h.numel();
  d.uniforms = static_cast<const float*>(row_param(uniforms, B, at::kFloat, x, "uniforms", keep));
  d.temperature = static_cast<const float*>(row_param(temperature, B, at::kFloat, x, "temperature", keep));
  d.top_k = static_cast<const int32_t*>(row_param(top_k, B, at::kInt, x, "top_k", keep));
  d.top_p = static_cast<const float*>(row_param(top_p, B, at::kFloat, x, "top_p", keep));
  d.penalty = static_cast<const float*>(row_param(penalty, B, at::kFloat, x, "penalty", keep));
  d.min_new_tokens = static_cast<const int32_t*>(row_param(min_new_tokens, B, at::kInt, x, "min_new_tokens", keep));
  if (suppress_mask.has_value()) {
    same_device(*suppress_mask, x, "suppress_mask");
    Tensor m = suppress_mask->reshape({-1}).to(at::kBool).contiguous();
    TORCH_CHECK(m.numel() == V, "q3s: suppress_mask has ", m.numel(), " entries for vocab ", V);
    keep.push_back(m);
    d.suppress_mask = reinterpret_cast<const uint8_t*>(m.data_ptr<bool>());
  }
  d.eos_id = static_cast<int32_t>(eos_id);
  Tensor ids = at::empty({B}, x.options().dtype(at::kLong));
  d.ids_i64 = ids.data_ptr<int64_t>();
  launch(d, x);
  return ids;
}

Tensor sample_cp_stage(const Tensor& logits, const c10::optional<Tensor>& temperature,
                       const c10::optional<Tensor>& gumbel_noise, int64_t topk) {
  const Tensor x = rows_2d(logits);
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.size(0), V = x.size(1);
  std::vector<Tensor> keep;
  q3s_sample_desc d = base_desc(x, Q3S_DRAW_GUMBEL);
  d.topk = static_cast<int32_t>(std::min<int64_t>(topk, V));
  if (gumbel_noise.has_value()) {  // else: argmax over the whole row (utils.py:1185-1186)
    same_device(*gumbel_noise, x, "gumbel_noise");
    Tensor g = gumbel_noise->reshape({B, -1});
    if (g.scalar_type() != at::kFloat || g.stride(1) != 1) g = g.to(at::kFloat).contiguous();
    TORCH_CHECK(g.size(1) >= d.topk, "q3s: gumbel_noise has ", g.size(1), " columns, need ", d.topk);
    keep.push_back(g);
    d.gumbel_noise = g.data_ptr<float>();
    d.gumbel_row_stride = B > 1 ? g.stride(0) : g.size(1);
    if (temperature.has_value())
      d.temperature = static_cast<const float*>(row_param(*temperature, B, at::kFloat, x, "temperature", keep));
  }
  Tensor ids = at::empty({B}, x.options().dtype(at::kLong));
  d.ids_i64 = ids.data_ptr<int64_t>();
  launch(d, x);
  return ids;
}

Tensor sample_cp_frame(const Tensor& logits, const Tensor& temperature, const c10::optional<Tensor>& cp_gumbel_noise,
                       int64_t topk) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 3, "q3s: cp frame logits must be a CUDA [S,B,V] tensor");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat,
              "q3s: logits must be bf16 or fp32");
  Tensor x = logits.stride(2) == 1 ? logits : logits.contiguous();
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t S = x.size(0), B = x.size(1), V = x.size(2);
  std::vector<Tensor> keep;
  q3s_cp_frame_desc d;
  std::memset(&d, 0, sizeof(d));
  d.struct_size = sizeof(q3s_cp_frame_desc);
  d.mode = Q3S_DRAW_GUMBEL;
  d.batch = static_cast<int32_t>(B);
  d.vocab = static_cast<int32_t>(V);
  d.stages = static_cast<int32_t>(S);
  d.topk = static_cast<int32_t>(std::min<int64_t>(topk, V));
  d.logits_dtype = dtype_code(x);
  d.producer = Q3S_CP_DIRECT;
  d.logits = x.data_ptr();
  d.logits_row_stride = B > 1 ? x.stride(1) : V;
  d.logits_stage_stride = S > 1 ? x.stride(0) : B * V;
  d.temperature_default = 1.0f;
  d.top_p_default = 1.0f;
  d.temperature = static_cast<const float*>(row_param(temperature, B, at::kFloat, x, "temperature", keep));
  if (cp_gumbel_noise.has_value()) {  // [B, S, >=K]; none: greedy per stage
    same_device(*cp_gumbel_noise, x, "cp_gumbel_noise");
    TORCH_CHECK(cp_gumbel_noise->dim() == 3 && cp_gumbel_noise->size(0) == B && cp_gumbel_noise->size(1) == S,
                "q3s: cp_gumbel_noise must be [B,S,K]");
    Tensor g = cp_gumbel_noise->to(at::kFloat).contiguous();
    TORCH_CHECK(g.size(2) >= d.topk, "q3s: cp_gumbel_noise has ", g.size(2), " columns, need ", d.topk);
    keep.push_back(g);
    d.gumbel_noise = g.data_ptr<float>();
    d.gumbel_row_stride = g.stride(0);
    d.gumbel_stage_stride = g.stride(1);
  }
  Tensor ids = at::empty({B, S}, x.options().dtype(at::kLong));
  d.ids_out = ids.data_ptr<int64_t>();
  check_status(q3s_sample_cp_frame(&d, c10::cuda::getCurrentCUDAStream(x.get_device()).stream()),
               "q3s_sample_cp_frame");
  return ids;
}

// ---- Meta kernels: shapes and dtypes only (tracing, torch.compile's fake tensors)
at::IntArrayRef::value_type batch_of(const Tensor& logits) { return logits.size(0); }

std::tuple<Tensor, Tensor> sample_codebook0_meta(const Tensor& logits, const Tensor& token_counts, const Tensor&,
                                                 const Tensor&, const Tensor&, const c10::optional<Tensor>&,
                                                 int64_t) {
  return {at::empty({batch_of(logits)}, logits.options().dtype(at::kLong)), at::empty_like(token_counts)};
}

Tensor sample_codebook0__meta(const Tensor& logits, Tensor&, const Tensor&, const Tensor&, const Tensor&,
                              const c10::optional<Tensor>&, int64_t) {
  return at::empty({batch_of(logits)}, logits.options().dtype(at::kLong));
}

Tensor sample_codebook0_packed_meta(const Tensor& logits, const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                    const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                    const c10::optional<Tensor>&, int64_t) {
  return at::empty({batch_of(logits)}, logits.options().dtype(at::kLong));
}

Tensor sample_cp_stage_meta(const Tensor& logits, const c10::optional<Tensor>&, const c10::optional<Tensor>&,
                            int64_t) {
  return at::empty({batch_of(logits)}, logits.options().dtype(at::kLong));
}

Tensor sample_cp_frame_meta(const Tensor& logits, const Tensor&, const c10::optional<Tensor>&, int64_t) {
  return at::empty({logits.size(1), logits.size(0)}, logits.options().dtype(at::kLong));
}

}  // namespace

TORCH_LIBRARY(q3s, m) {
  m.def("sample_codebook0(Tensor logits, Tensor token_counts, Tensor gumbel_noise, Tensor temperature, "
        "Tensor penalty, Tensor? suppress_mask=None, int topk=50) -> (Tensor, Tensor)");
  m.def("sample_codebook0_(Tensor logits, Tensor(a!) token_counts, Tensor gumbel_noise, Tensor temperature, "
        "Tensor penalty, Tensor? suppress_mask=None, int topk=50) -> Tensor");
  m.def("sample_codebook0_packed(Tensor logits, Tensor history, Tensor offsets, Tensor uniforms, "
        "Tensor temperature, Tensor top_k, Tensor top_p, Tensor penalty, Tensor min_new_tokens, "
        "Tensor? suppress_mask=None, int eos_id=2150) -> Tensor");
  m.def("sample_cp_stage(Tensor logits, Tensor? temperature=None, Tensor? gumbel_noise=None, int topk=50) -> Tensor");
  m.def("sample_cp_frame(Tensor logits, Tensor temperature, Tensor? cp_gumbel_noise=None, int topk=50) -> Tensor");
}

TORCH_LIBRARY_IMPL(q3s, CUDA, m) {
  m.impl("sample_codebook0", &sample_codebook0);
  m.impl("sample_codebook0_", &sample_codebook0_);
  m.impl("sample_codebook0_packed", &sample_codebook0_packed);
  m.impl("sample_cp_stage", &sample_cp_stage);
  m.impl("sample_cp_frame", &sample_cp_frame);
}

TORCH_LIBRARY_IMPL(q3s, Meta, m) {
  m.impl("sample_codebook0", &sample_codebook0_meta);
  m.impl("sample_codebook0_", &sample_codebook0__meta);
  m.impl("sample_codebook0_packed", &sample_codebook0_packed_meta);
  m.impl("sample_cp_stage", &sample_cp_stage_meta);
  m.impl("sample_cp_frame", &sample_cp_frame_meta);
}
