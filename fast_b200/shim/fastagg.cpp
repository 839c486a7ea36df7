// Drop-in `fastAgg` module: the reference operator names, argument order,
// dtypes and list-of-tensor returns (NoneBone/FAST
// getFastAgg/cuda_operators/operators.cpp:606-624), implemented over the
// libfast_b200 C ABI.  Differences from the reference, all deliberate:
//   * kernels run on torch's current CUDA stream and never synchronise; the
//     reference's per-call cudaDeviceSynchronize and NaN-check device->host
//     copies (operators.cpp:184-203) are gone;
//   * forward_tgat / backward_tgat aggregate every edge (the reference grid
//     only covers ceil8(dst_num) edges, aggregate_acc_kernel.cu:47-48,82-92);
//   * backward_tgat_shd returns dv[col] = dy[row] (the reference sums dy over
//     the segment, scaling the gradient by the in-degree, aggregate_shd_kernel.cu:343-364);
//   * forward_fused_attn treats a segment's edges as [indptr[s], indptr[s+1])
//     (the reference indexes them through `indices`, which its caller fills
//     with the segment pointer itself, layers.py:190);
//   * kernel errors raise RuntimeError instead of being printed.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <string>
#include <vector>

#include "fast_b200.h"

namespace {

#define CHECK_INPUT(x)                                                    \
  TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor");                \
  TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_DTYPE(x, t) TORCH_CHECK((x).scalar_type() == (t), #x " has the wrong dtype")

void check(int rc) {
  if (rc != FB_OK) throw std::runtime_error(std::string("fast_b200: ") + fb_last_error());
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

torch::TensorOptions f32(const torch::Tensor &like) {
  return torch::TensorOptions().dtype(torch::kFloat32).device(like.device());
}

using TL = std::vector<torch::Tensor>;

// ---- edge softmax (K1-K4) ---------------------------------------------------
TL edge_softmax_fwd_impl(torch::Tensor indptr, torch::Tensor x, int heads) {
  CHECK_INPUT(indptr); CHECK_INPUT(x);
  CHECK_DTYPE(indptr, torch::kInt32); CHECK_DTYPE(x, torch::kFloat32);
  TORCH_CHECK(x.dim() == 2 && x.size(1) == heads, "input_feat must be [E, num_heads]");
  const at::cuda::CUDAGuard g(x.device());
  auto y = torch::zeros({x.size(0), heads}, f32(x));
  check(fb_edge_softmax_fwd(indptr.data_ptr<int32_t>(), indptr.size(0) - 1, x.data_ptr<float>(), heads,
                            y.data_ptr<float>(), cur_stream()));
  return {y};
}

TL edge_softmax_bwd_impl(torch::Tensor indptr, torch::Tensor dy, torch::Tensor y) {
  CHECK_INPUT(indptr); CHECK_INPUT(dy); CHECK_INPUT(y);
  CHECK_DTYPE(indptr, torch::kInt32); CHECK_DTYPE(dy, torch::kFloat32); CHECK_DTYPE(y, torch::kFloat32);
  TORCH_CHECK(dy.sizes() == y.sizes() && dy.dim() == 2, "d_output and output must both be [E, heads]");
  const at::cuda::CUDAGuard g(dy.device());
  auto dx = torch::zeros_like(dy);
  check(fb_edge_softmax_bwd(indptr.data_ptr<int32_t>(), indptr.size(0) - 1, dy.data_ptr<float>(),
                            y.data_ptr<float>(), (int)dy.size(1), dx.data_ptr<float>(), cur_stream()));
  return {dx};
}

TL forward_edge_softmax(torch::Tensor indptr, torch::Tensor indices, torch::Tensor input_feat,
                        int node_num_per_block, int num_heads) {
  CHECK_INPUT(indices);
  return edge_softmax_fwd_impl(indptr, input_feat, num_heads);
}

TL backward_edge_softmax(torch::Tensor indptr, torch::Tensor indices, torch::Tensor d_output, torch::Tensor output,
                         int node_num_per_block, int num_heads) {
  CHECK_INPUT(indices);
  return edge_softmax_bwd_impl(indptr, d_output, output);
}

TL forward_csr_edge_softmax(torch::Tensor indptr, torch::Tensor indices, torch::Tensor input_feat,
                            int node_num_per_block, int reduce_size) {
  CHECK_INPUT(indices);
  return edge_softmax_fwd_impl(indptr, input_feat, (int)input_feat.size(1));
}

TL backward_csr_edge_softmax(torch::Tensor indptr, torch::Tensor indices, torch::Tensor d_output,
                             torch::Tensor output, int node_num_per_block, int reduce_size) {
  CHECK_INPUT(indices);
  return edge_softmax_bwd_impl(indptr, d_output, output);
}

TL forward_balanced_edge_softmax(torch::Tensor, torch::Tensor, torch::Tensor, int, int) {
  throw std::runtime_error(
      "fast_b200: forward_balanced_edge_softmax is not provided (never called by the reference; "
      "use forward_edge_softmax)");
}

TL backward_balanced_edge_softmax(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int, int) {
  throw std::runtime_error(
      "fast_b200: backward_balanced_edge_softmax is not provided (never called by the reference; "
      "use backward_edge_softmax)");
}

// ---- aggregation (K7-K10) ---------------------------------------------------
TL scatter_impl(torch::Tensor dst_idx, torch::Tensor src_idx, torch::Tensor v, int64_t n_out) {
  CHECK_INPUT(dst_idx); CHECK_INPUT(src_idx); CHECK_INPUT(v);
  CHECK_DTYPE(dst_idx, torch::kInt64); CHECK_DTYPE(src_idx, torch::kInt64); CHECK_DTYPE(v, torch::kFloat32);
  TORCH_CHECK(v.dim() == 2, "feature input must be 2-D");
  TORCH_CHECK(dst_idx.numel() == src_idx.numel(), "edge index lists differ in length");
  const at::cuda::CUDAGuard g(v.device());
  auto out = torch::zeros({n_out, v.size(1)}, f32(v));
  check(fb_scatter_rows(dst_idx.data_ptr<int64_t>(), src_idx.data_ptr<int64_t>(), dst_idx.numel(),
                        v.data_ptr<float>(), v.size(0), (int)v.size(1), out.data_ptr<float>(), n_out, cur_stream()));
  return {out};
}

TL forward_tgat(torch::Tensor src_edges, torch::Tensor dst_edges, torch::Tensor input_feat, int dst_num,
                int aggNodePB, int aggFeat) {
  return scatter_impl(src_edges, dst_edges, input_feat, dst_num);
}

TL backward_tgat(torch::Tensor src_edges, torch::Tensor dst_edges, torch::Tensor d_input, int src_num,
                 int aggNodePB, int aggFeat) {
  return scatter_impl(dst_edges, src_edges, d_input, src_num);
}

TL forward_tgat_shd(torch::Tensor indptr, torch::Tensor indices, torch::Tensor src_edges, torch::Tensor dst_edges,
                    torch::Tensor input_feat, int dst_nodes, int aggNodePB, int aggFeat) {
  CHECK_INPUT(indptr); CHECK_INPUT(indices); CHECK_INPUT(src_edges); CHECK_INPUT(dst_edges); CHECK_INPUT(input_feat);
  CHECK_DTYPE(indptr, torch::kInt32); CHECK_DTYPE(src_edges, torch::kInt64); CHECK_DTYPE(dst_edges, torch::kInt64);
  CHECK_DTYPE(input_feat, torch::kFloat32);
  const at::cuda::CUDAGuard g(input_feat.device());
  auto out = torch::zeros({(int64_t)dst_nodes, input_feat.size(1)}, f32(input_feat));
  check(fb_segment_rows(indptr.data_ptr<int32_t>(), indptr.size(0) - 1, src_edges.data_ptr<int64_t>(),
                        dst_edges.data_ptr<int64_t>(), input_feat.data_ptr<float>(), input_feat.size(0),
                        (int)input_feat.size(1), out.data_ptr<float>(), dst_nodes, cur_stream()));
  return {out};
}

// Argument names follow operators.cpp:337-345; the reference caller passes the
// destination-row list first and the source list second (efficientGOP.py:126).
TL backward_tgat_shd(torch::Tensor indptr, torch::Tensor indices, torch::Tensor dst_edges, torch::Tensor src_edges,
                     torch::Tensor d_input, int src_nodes, int aggNodePB, int aggFeat) {
  CHECK_INPUT(indptr); CHECK_INPUT(indices);
  return scatter_impl(src_edges, dst_edges, d_input, src_nodes);
}

// ---- fused attention over precomputed logits (K11/K12) ----------------------
TL forward_fused_attn(torch::Tensor input_feat, torch::Tensor V_val, torch::Tensor indptr, torch::Tensor indices,
                      torch::Tensor dst_eid, torch::Tensor src_eid, int node_num, int num_heads,
                      double negative_slope, double attn_drop) {
  CHECK_INPUT(input_feat); CHECK_INPUT(V_val); CHECK_INPUT(indptr); CHECK_INPUT(dst_eid);
  CHECK_DTYPE(input_feat, torch::kFloat32); CHECK_DTYPE(V_val, torch::kFloat32);
  CHECK_DTYPE(indptr, torch::kInt32); CHECK_DTYPE(dst_eid, torch::kInt64);
  TORCH_CHECK(V_val.dim() == 3 && V_val.size(1) == num_heads && input_feat.size(1) == num_heads,
              "V_val must be [E, heads, D/heads] and input_feat [E, heads]");
  const at::cuda::CUDAGuard g(V_val.device());
  const int64_t E = input_feat.size(0);
  const int dim = (int)(V_val.size(1) * V_val.size(2));
  auto att = torch::zeros({E, (int64_t)num_heads}, f32(V_val));
  auto agg = torch::zeros({(int64_t)node_num, (int64_t)dim}, f32(V_val));
  auto mask = torch::rand({E, (int64_t)num_heads}, f32(V_val));
  check(fb_attn_logits_fwd(input_feat.data_ptr<float>(), V_val.data_ptr<float>(), dim, indptr.data_ptr<int32_t>(),
                           indptr.size(0) - 1, dst_eid.data_ptr<int64_t>(), (int64_t)node_num, num_heads, dim,
                           (float)negative_slope,
                           (float)attn_drop, mask.data_ptr<float>(), att.data_ptr<float>(), agg.data_ptr<float>(),
                           cur_stream()));
  return {agg, att, mask};
}

// Returns [d_logits, dV].  Without `input_feat` the logits gradient is taken
// with respect to the activated logits, as the reference computes it
// (fused_attention.cu:430-444); pass input_feat to include LeakyReLU'.
TL backward_fused_attn(torch::Tensor d_output, torch::Tensor V_val, torch::Tensor output_attn,
                       torch::Tensor edge_mask, torch::Tensor indptr, torch::Tensor indices, torch::Tensor dst_eid,
                       torch::Tensor src_eid, int node_num, int num_heads, double negative_slope, double attn_drop,
                       c10::optional<torch::Tensor> input_feat) {
  CHECK_INPUT(d_output); CHECK_INPUT(V_val); CHECK_INPUT(output_attn); CHECK_INPUT(edge_mask);
  CHECK_INPUT(indptr); CHECK_INPUT(dst_eid);
  CHECK_DTYPE(d_output, torch::kFloat32); CHECK_DTYPE(V_val, torch::kFloat32);
  const at::cuda::CUDAGuard g(V_val.device());
  const int64_t E = output_attn.size(0);
  const int dim = (int)(V_val.size(1) * V_val.size(2));
  auto dx = torch::zeros({E, (int64_t)num_heads}, f32(V_val));
  auto dv = torch::zeros_like(V_val);
  const float *x = nullptr;
  torch::Tensor xin;
  float slope = (float)negative_slope;
  if (input_feat.has_value()) {
    xin = input_feat.value();
    CHECK_INPUT(xin);
    x = xin.data_ptr<float>();
  } else {
    // Without the logits the activation is treated as the identity.
    xin = torch::ones({E, (int64_t)num_heads}, f32(V_val));
    x = xin.data_ptr<float>();
    slope = 1.f;
  }
  check(fb_attn_logits_bwd(x, V_val.data_ptr<float>(), dim, indptr.data_ptr<int32_t>(), indptr.size(0) - 1,
                           dst_eid.data_ptr<int64_t>(), d_output.size(0), num_heads, dim, slope, (float)attn_drop,
                           edge_mask.data_ptr<float>(), output_attn.data_ptr<float>(), d_output.data_ptr<float>(),
                           dx.data_ptr<float>(), dv.data_ptr<float>(), cur_stream()));
  return {dx, dv};
}

// ---- fused q.k -> softmax -> aggregate (new fast path) ----------------------
void check_rows(const torch::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.stride(1) == 1, name, " must be a 2-D CUDA tensor with unit column stride");
  CHECK_DTYPE(t, torch::kFloat32);
}

// q [Nd, D] (or [1, D] broadcast), k/v [E, D] rows (views into one [E, 2D]
// buffer allowed), rptr [Nd+1] CSR over destinations.  Returns [agg, att].
TL forward_fused_softmax_agg(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor rptr, int num_heads,
                             double negative_slope, double attn_drop, int64_t seed, int64_t offset) {
  check_rows(q, "q"); check_rows(k, "k"); check_rows(v, "v");
  CHECK_INPUT(rptr); CHECK_DTYPE(rptr, torch::kInt32);
  TORCH_CHECK(k.stride(0) == v.stride(0) && k.sizes() == v.sizes(), "k and v must share shape and row stride");
  const at::cuda::CUDAGuard g(q.device());
  const int64_t nd = rptr.size(0) - 1, E = k.size(0);
  const int dim = (int)k.size(1);
  const int64_t ldq = (q.size(0) == 1 && nd != 1) ? 0 : q.stride(0);
  TORCH_CHECK(ldq == 0 || q.size(0) == nd, "q must have one row per destination (or one row to broadcast)");
  auto att = torch::empty({E, (int64_t)num_heads}, f32(q));
  auto agg = torch::empty({nd, (int64_t)dim}, f32(q));
  check(fb_attn_fwd(q.data_ptr<float>(), ldq, k.data_ptr<float>(), v.data_ptr<float>(), k.stride(0),
                    rptr.data_ptr<int32_t>(), nd, nullptr, num_heads, dim, (float)negative_slope, (float)attn_drop,
                    (uint64_t)seed, (uint64_t)offset, nullptr, att.data_ptr<float>(), agg.data_ptr<float>(), dim,
                    cur_stream()));
  return {agg, att};
}

// Returns [dq (per destination), dk, dv].
TL backward_fused_softmax_agg(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor rptr,
                              torch::Tensor att, torch::Tensor dagg, int num_heads, double negative_slope,
                              double attn_drop, int64_t seed, int64_t offset) {
  check_rows(q, "q"); check_rows(k, "k"); check_rows(v, "v"); check_rows(dagg, "dagg");
  CHECK_INPUT(rptr); CHECK_INPUT(att);
  const at::cuda::CUDAGuard g(q.device());
  const int64_t nd = rptr.size(0) - 1, E = k.size(0);
  const int dim = (int)k.size(1);
  const int64_t ldq = (q.size(0) == 1 && nd != 1) ? 0 : q.stride(0);
  auto dq = torch::empty({nd, (int64_t)dim}, f32(q));
  auto dk = torch::empty({E, (int64_t)dim}, f32(q));
  auto dv = torch::empty({E, (int64_t)dim}, f32(q));
  check(fb_attn_bwd(q.data_ptr<float>(), ldq, k.data_ptr<float>(), v.data_ptr<float>(), k.stride(0),
                    rptr.data_ptr<int32_t>(), nd, nullptr, num_heads, dim, (float)negative_slope, (float)attn_drop,
                    (uint64_t)seed, (uint64_t)offset, nullptr, att.data_ptr<float>(), dagg.data_ptr<float>(),
                    dagg.stride(0),
                    dq.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>(), dim, cur_stream()));
  return {dq, dk, dv};
}

// ---- utils (utils.cu) -------------------------------------------------------
torch::Tensor exclusive_sum(torch::Tensor in_degs) {
  CHECK_INPUT(in_degs); CHECK_DTYPE(in_degs, torch::kInt32);
  const at::cuda::CUDAGuard g(in_degs.device());
  const int64_t n = in_degs.numel();
  auto out = torch::empty({n + 1}, in_degs.options());
  auto ws = torch::empty({(int64_t)fb_exclusive_sum_ws_bytes(n)}, in_degs.options().dtype(torch::kUInt8));
  check(fb_exclusive_sum(in_degs.data_ptr<int32_t>(), n, out.data_ptr<int32_t>(), ws.data_ptr(), cur_stream()));
  return out;
}

torch::Tensor cal_deg(torch::Tensor edges, int nodes_num) {
  CHECK_INPUT(edges); CHECK_DTYPE(edges, torch::kInt32);
  const at::cuda::CUDAGuard g(edges.device());
  auto deg = torch::zeros({(int64_t)nodes_num}, edges.options());
  check(fb_count_ids(edges.data_ptr<int32_t>(), edges.numel(), deg.data_ptr<int32_t>(), nodes_num, cur_stream()));
  return deg;
}

torch::Tensor getBalancedPtr(torch::Tensor densePtr, int threshold) {
  CHECK_INPUT(densePtr); CHECK_DTYPE(densePtr, torch::kInt32);
  TORCH_CHECK(densePtr.numel() >= 1, "densePtr must not be empty");
  const at::cuda::CUDAGuard g(densePtr.device());
  auto mask = torch::zeros({densePtr.numel() - 1}, densePtr.options());
  check(fb_balanced_mask(densePtr.data_ptr<int32_t>(), densePtr.numel(), threshold, mask.data_ptr<int32_t>(),
                         cur_stream()));
  return mask;
}

}  // namespace

PYBIND11_MODULE(fastAgg, m) {
  m.doc() = "fast_b200 drop-in for the FAST fastAgg CUDA operators (sm_100a)";
  m.def("cal_deg", &cal_deg, "cal_deg (CUDA)");
  m.def("exclusive_sum", &exclusive_sum, "exclusive_sum (CUDA)");
  m.def("getBalancedPtr", &getBalancedPtr, "balanced_ptr (CUDA)");
  m.def("forward_tgat", &forward_tgat, "scatter-sum aggregate (CUDA)");
  m.def("backward_tgat", &backward_tgat, "scatter-sum aggregate backward (CUDA)");
  m.def("forward_edge_softmax", &forward_edge_softmax, "edge softmax (CUDA)");
  m.def("backward_edge_softmax", &backward_edge_softmax, "edge softmax backward (CUDA)");
  m.def("forward_tgat_shd", &forward_tgat_shd, "segment aggregate (CUDA)");
  m.def("backward_tgat_shd", &backward_tgat_shd, "segment aggregate backward (CUDA)");
  m.def("forward_balanced_edge_softmax", &forward_balanced_edge_softmax, "not provided");
  m.def("backward_balanced_edge_softmax", &backward_balanced_edge_softmax, "not provided");
  m.def("forward_csr_edge_softmax", &forward_csr_edge_softmax, "edge softmax, any degree (CUDA)");
  m.def("backward_csr_edge_softmax", &backward_csr_edge_softmax, "edge softmax backward, any degree (CUDA)");
  m.def("forward_fused_attn", &forward_fused_attn, "LeakyReLU + softmax + dropout + aggregate (CUDA)");
  m.def("backward_fused_attn", &backward_fused_attn, "backward of forward_fused_attn (CUDA)",
        py::arg("d_output"), py::arg("V_val"), py::arg("output_attn"), py::arg("edge_mask"), py::arg("indptr"),
        py::arg("indices"), py::arg("dst_eid"), py::arg("src_eid"), py::arg("node_num"), py::arg("num_heads"),
        py::arg("negative_slope"), py::arg("attn_drop"), py::arg("input_feat") = py::none());
  m.def("forward_fused_softmax_agg", &forward_fused_softmax_agg, "q.k -> edge softmax -> aggregate in one kernel");
  m.def("backward_fused_softmax_agg", &backward_fused_softmax_agg, "backward of forward_fused_softmax_agg");
}
