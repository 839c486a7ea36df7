// Drop-in `sampler_core` module: ParallelSampler / TemporalGraphBlock with the
// reference's constructor arguments, methods and numpy-returning accessors
// (NoneBone/FAST getSamplerCore/sampler_core.cpp:1115-1149), backed by the
// device sampler of libfast_b200.  The CSR and the time pointers live in HBM;
// sample() enqueues every layer on torch's current stream.
//
// Additions for the device-resident training path:
//   ParallelSampler.sample_device(roots, ts)   roots/ts already on the GPU
//   ParallelSampler.sample_shard(roots, ts, global_roots, global_ts)
//                                              one data-parallel rank's roots,
//                                              pointers advanced by the global batch
//   ParallelSampler.block_views()              zero-copy device views (valid
//                                              until the next sample call)
//   ParallelSampler.dims()                     per-block sizes (synchronises)
//   TemporalGraphBlock.<name>_t()              device tensors of get_ret() blocks
// OpenMP affinity controls (configOMP, clear_cpu_affinity, check_bind) are
// accepted and ignored: the device sampler has no host threads to pin.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>

#include <chrono>
#include <memory>
#include <string>
#include <vector>

#include "fast_b200.h"

namespace py = pybind11;

namespace {

void check(int rc) {
  if (rc != FB_OK) throw std::runtime_error(std::string("fast_b200 sampler: ") + fb_last_error());
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

struct Handle {
  fb_sampler *s = nullptr;
  int device = 0;
  std::vector<torch::Tensor> keep;  // borrowed device graph
  ~Handle() {
    if (s) fb_sampler_destroy(s);
  }
};

py::array tensor_to_numpy(const torch::Tensor &t) {
  torch::Tensor c = t.to(torch::kCPU).contiguous();
  if (c.scalar_type() == torch::kInt32) {
    py::array_t<int32_t> a(c.numel());
    if (c.numel()) std::memcpy(a.mutable_data(), c.data_ptr<int32_t>(), c.numel() * 4);
    return a;
  }
  py::array_t<float> a(c.numel());
  if (c.numel()) std::memcpy(a.mutable_data(), c.data_ptr<float>(), c.numel() * 4);
  return a;
}

// View `n` elements at `p` as a device tensor that keeps the sampler alive.
torch::Tensor view_of(const std::shared_ptr<Handle> &h, void *p, int64_t n, torch::ScalarType t) {
  auto keep = h;
  auto opts = torch::TensorOptions().dtype(t).device(torch::kCUDA, h->device);
  return torch::from_blob(p, {n}, [keep](void *) {}, opts);
}

class Block {
 public:
  torch::Tensor row, col, eid, ts, dts, nodes, uniE, invE, cntE, rptr;
  int64_t dim_in = 0, dim_out = 0;
  double tot = 0, ptr = 0, search = 0, sample = 0, coo = 0;

  Block() = default;
  // Host-side constructor with the reference signature (sampler_core.cpp:1118-1122).
  Block(std::vector<int32_t> r, std::vector<int32_t> c, std::vector<int32_t> e, std::vector<float> t,
        std::vector<float> d, std::vector<int32_t> n, std::vector<int32_t> u, std::vector<int32_t> i,
        std::vector<int32_t> ce, int32_t din, int32_t dout) {
    auto I = [](const std::vector<int32_t> &v) { return torch::tensor(v, torch::kInt32); };
    auto F = [](const std::vector<float> &v) { return torch::tensor(v, torch::kFloat32); };
    row = I(r); col = I(c); eid = I(e); ts = F(t); dts = F(d); nodes = I(n); uniE = I(u); invE = I(i); cntE = I(ce);
    dim_in = din; dim_out = dout;
  }
};

class Sampler {
 public:
  std::shared_ptr<Handle> h;
  int num_layers, num_history;
  std::vector<int> uni_flag;
  double last_tot = 0;

  Sampler(py::object indptr, py::object indices, py::object eid, py::object ts, int num_thread_per_worker,
          int num_workers, int num_layers_, std::vector<int> num_neighbors, bool recent, bool prop_time,
          int num_history_, float window_duration, uint64_t seed)
      : num_layers(num_layers_), num_history(num_history_) {
    TORCH_CHECK((int)num_neighbors.size() >= num_layers_, "num_neighbors needs one entry per layer");
    h = std::make_shared<Handle>();
    std::vector<int32_t> nn(num_neighbors.begin(), num_neighbors.end());
    bool on_dev = false;
    if (THPVariable_Check(indptr.ptr())) {
      torch::Tensor ip = THPVariable_Unpack(indptr.ptr());
      on_dev = ip.is_cuda();
    }
    if (on_dev) {
      auto T = [](py::object o) { return THPVariable_Unpack(o.ptr()).contiguous(); };
      torch::Tensor ip = T(indptr), ix = T(indices), ei = T(eid), t = T(ts);
      TORCH_CHECK(ip.scalar_type() == torch::kInt32 && ix.scalar_type() == torch::kInt32 &&
                      ei.scalar_type() == torch::kInt32 && t.scalar_type() == torch::kFloat32,
                  "device graph: indptr/indices/eid int32, ts float32");
      h->device = ip.get_device();
      const c10::cuda::CUDAGuard g(h->device);
      h->keep = {ip, ix, ei, t};
      check(fb_sampler_create(ip.data_ptr<int32_t>(), ix.data_ptr<int32_t>(), ei.data_ptr<int32_t>(),
                              t.data_ptr<float>(), ip.numel() - 1, ix.numel(), 1, num_layers, nn.data(), recent,
                              prop_time, num_history, window_duration, seed, &h->s));
    } else {
      using AI = py::array_t<int32_t, py::array::c_style | py::array::forcecast>;
      using AF = py::array_t<float, py::array::c_style | py::array::forcecast>;
      AI ip = AI::ensure(indptr), ix = AI::ensure(indices), ei = AI::ensure(eid);
      AF t = AF::ensure(ts);
      TORCH_CHECK(ip && ix && ei && t, "graph arrays must convert to int32/float32 numpy arrays");
      TORCH_CHECK(ix.size() == ei.size() && ix.size() == t.size(), "indices/eid/ts lengths differ");
      h->device = c10::cuda::current_device();
      const c10::cuda::CUDAGuard g(h->device);
      check(fb_sampler_create(ip.data(), ix.data(), ei.data(), t.data(), ip.size() - 1, ix.size(), 0, num_layers,
                              nn.data(), recent, prop_time, num_history, window_duration, seed, &h->s));
    }
    uni_flag.assign(num_layers * num_history, 1);
  }

  void reset() {
    const c10::cuda::CUDAGuard g(h->device);
    check(fb_sampler_reset(h->s, cur_stream()));
  }

  void apply_flags(const std::vector<int> &csr_flag) {
    std::fill(uni_flag.begin(), uni_flag.end(), 1);
    // Only the first block honours the flag, as in sampler_core.cpp:693-696.
    if (csr_flag.size() >= 3 && !uni_flag.empty()) uni_flag[0] = csr_flag[0];
  }

  void sample(py::array_t<int32_t, py::array::c_style | py::array::forcecast> roots,
              py::array_t<float, py::array::c_style | py::array::forcecast> root_ts, std::vector<int> csr_flag) {
    TORCH_CHECK(roots.size() == root_ts.size(), "roots and ts differ in length");
    const c10::cuda::CUDAGuard g(h->device);
    auto t0 = std::chrono::steady_clock::now();
    apply_flags(csr_flag);
    check(fb_sampler_sample(h->s, roots.data(), root_ts.data(), roots.size(), 0, cur_stream()));
    last_tot = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }

  void sample_device(torch::Tensor roots, torch::Tensor root_ts) {
    TORCH_CHECK(roots.is_cuda() && root_ts.is_cuda() && roots.is_contiguous() && root_ts.is_contiguous(),
                "sample_device wants contiguous CUDA tensors");
    TORCH_CHECK(roots.scalar_type() == torch::kInt32 && root_ts.scalar_type() == torch::kFloat32,
                "roots int32, ts float32");
    TORCH_CHECK(roots.numel() == root_ts.numel(), "roots and ts differ in length");
    const c10::cuda::CUDAGuard g(h->device);
    check(fb_sampler_sample(h->s, roots.data_ptr<int32_t>(), root_ts.data_ptr<float>(), roots.numel(), 1,
                            cur_stream()));
  }

  // Pointer updates of the first layer for (global) device roots, no sampling.
  void update_pointers(torch::Tensor roots, torch::Tensor root_ts) {
    TORCH_CHECK(roots.is_cuda() && root_ts.is_cuda() && roots.is_contiguous() && root_ts.is_contiguous(),
                "update_pointers wants contiguous CUDA tensors");
    TORCH_CHECK(roots.scalar_type() == torch::kInt32 && root_ts.scalar_type() == torch::kFloat32,
                "roots int32, ts float32");
    TORCH_CHECK(roots.numel() == root_ts.numel(), "roots and ts differ in length");
    const c10::cuda::CUDAGuard g(h->device);
    check(fb_sampler_update_pointers(h->s, roots.data_ptr<int32_t>(), root_ts.data_ptr<float>(), roots.numel(),
                                     cur_stream()));
  }

  // One data-parallel rank's sample(): its own device roots, with the time
  // pointers advanced as one sample() over the global batch's roots would.
  void sample_shard(torch::Tensor roots, torch::Tensor root_ts, torch::Tensor global_roots,
                    torch::Tensor global_ts) {
    for (const auto *t : {&roots, &root_ts, &global_roots, &global_ts})
      TORCH_CHECK(t->is_cuda() && t->is_contiguous(), "sample_shard wants contiguous CUDA tensors");
    TORCH_CHECK(roots.scalar_type() == torch::kInt32 && global_roots.scalar_type() == torch::kInt32 &&
                    root_ts.scalar_type() == torch::kFloat32 && global_ts.scalar_type() == torch::kFloat32,
                "roots int32, ts float32");
    TORCH_CHECK(roots.numel() == root_ts.numel() && global_roots.numel() == global_ts.numel(),
                "roots and ts differ in length");
    const c10::cuda::CUDAGuard g(h->device);
    check(fb_sampler_sample_shard(h->s, roots.data_ptr<int32_t>(), root_ts.data_ptr<float>(), roots.numel(),
                                  global_roots.data_ptr<int32_t>(), global_ts.data_ptr<float>(),
                                  global_roots.numel(), cur_stream()));
  }

  std::vector<std::vector<int32_t>> dims() {
    const c10::cuda::CUDAGuard g(h->device);
    const int nb = fb_sampler_num_blocks(h->s);
    std::vector<int32_t> host(8 * nb);
    check(fb_sampler_dims(h->s, host.data(), cur_stream()));
    std::vector<std::vector<int32_t>> out(nb);
    for (int i = 0; i < nb; ++i) out[i].assign(host.begin() + 8 * i, host.begin() + 8 * i + 5);
    return out;
  }

  py::list block_views() {
    py::list out;
    const int nb = fb_sampler_num_blocks(h->s);
    for (int i = 0; i < nb; ++i) {
      fb_block_view v;
      check(fb_sampler_block(h->s, i, &v));
      const int64_t cr = v.max_roots, ce = std::max<int64_t>(v.max_edges, 1);
      py::dict d;
      d["row"] = view_of(h, v.row, ce, torch::kInt32);
      d["col"] = view_of(h, v.col, ce, torch::kInt32);
      d["eid"] = view_of(h, v.eid, ce, torch::kInt32);
      d["ts"] = view_of(h, v.ts, cr + ce, torch::kFloat32);
      d["dts"] = view_of(h, v.dts, cr + ce, torch::kFloat32);
      d["nodes"] = view_of(h, v.nodes, cr + ce, torch::kInt32);
      d["rptr"] = view_of(h, v.rptr, cr + 1, torch::kInt32);
      d["cntE"] = view_of(h, v.cntE, cr + 1, torch::kInt32);
      d["uniE"] = view_of(h, v.uniE, ce, torch::kInt32);
      d["invE"] = view_of(h, v.invE, ce, torch::kInt32);
      d["dims"] = view_of(h, v.dims, 8, torch::kInt32);
      d["dte"] = view_of(h, v.dte, ce, torch::kFloat32);
      d["nbr"] = view_of(h, v.nbr, ce, torch::kInt32);
      d["max_roots"] = cr;
      d["max_edges"] = v.max_edges;
      out.append(d);
    }
    return out;
  }

  void dedup(int i) {
    const c10::cuda::CUDAGuard g(h->device);
    check(fb_sampler_dedup(h->s, i, cur_stream()));
  }

  void set_call_index(uint64_t i) { check(fb_sampler_set_call_index(h->s, i)); }

  // ParallelSampler::get_ret: an owning copy of every block.
  std::vector<Block> get_ret() {
    const c10::cuda::CUDAGuard g(h->device);
    const int nb = fb_sampler_num_blocks(h->s);
    for (int i = 0; i < nb; ++i)
      if (uni_flag[i]) check(fb_sampler_dedup(h->s, i, cur_stream()));
    std::vector<int32_t> host(8 * nb);
    check(fb_sampler_dims(h->s, host.data(), cur_stream()));
    std::vector<Block> out(nb);
    for (int i = 0; i < nb; ++i) {
      fb_block_view v;
      check(fb_sampler_block(h->s, i, &v));
      const int32_t R = host[8 * i], E = host[8 * i + 1], S = host[8 * i + 2], nu = host[8 * i + 4];
      Block &b = out[i];
      auto cp = [&](void *p, int64_t n, torch::ScalarType t) {
        return n > 0 ? view_of(h, p, n, t).clone()
                     : torch::empty({0}, torch::TensorOptions().dtype(t).device(torch::kCUDA, h->device));
      };
      b.row = cp(v.row, E, torch::kInt32);
      b.col = cp(v.col, E, torch::kInt32);
      b.eid = cp(v.eid, E, torch::kInt32);
      b.ts = cp(v.ts, R + E, torch::kFloat32);
      b.dts = cp(v.dts, R + E, torch::kFloat32);
      b.nodes = cp(v.nodes, R + E, torch::kInt32);
      b.rptr = cp(v.rptr, R + 1, torch::kInt32);
      b.cntE = cp(v.cntE, E > 0 ? S + 1 : 0, torch::kInt32);
      b.uniE = cp(v.uniE, uni_flag[i] ? nu : 0, torch::kInt32);
      b.invE = cp(v.invE, uni_flag[i] ? E : 0, torch::kInt32);
      b.dim_in = R + E;
      b.dim_out = R;
      if (i == 0) b.tot = last_tot;
    }
    return out;
  }
};

}  // namespace

PYBIND11_MODULE(sampler_core, m) {
  m.doc() = "fast_b200 drop-in for the FAST temporal sampler (device-resident, sm_100a)";
  py::class_<Block>(m, "TemporalGraphBlock")
      .def(py::init<std::vector<int32_t>, std::vector<int32_t>, std::vector<int32_t>, std::vector<float>,
                    std::vector<float>, std::vector<int32_t>, std::vector<int32_t>, std::vector<int32_t>,
                    std::vector<int32_t>, int32_t, int32_t>())
      .def("row", [](const Block &b) { return tensor_to_numpy(b.row); })
      .def("col", [](const Block &b) { return tensor_to_numpy(b.col); })
      .def("eid", [](const Block &b) { return tensor_to_numpy(b.eid); })
      .def("ts", [](const Block &b) { return tensor_to_numpy(b.ts); })
      .def("dts", [](const Block &b) { return tensor_to_numpy(b.dts); })
      .def("nodes", [](const Block &b) { return tensor_to_numpy(b.nodes); })
      .def("uniE", [](const Block &b) { return tensor_to_numpy(b.uniE); })
      .def("invE", [](const Block &b) { return tensor_to_numpy(b.invE); })
      .def("cntE", [](const Block &b) { return tensor_to_numpy(b.cntE); })
      .def("dim_in", [](const Block &b) { return b.dim_in; })
      .def("dim_out", [](const Block &b) { return b.dim_out; })
      .def("tot_time", [](const Block &b) { return b.tot; })
      .def("ptr_time", [](const Block &b) { return b.ptr; })
      .def("search_time", [](const Block &b) { return b.search; })
      .def("sample_time", [](const Block &b) { return b.sample; })
      .def("coo_time", [](const Block &b) { return b.coo; })
      .def("row_t", [](const Block &b) { return b.row; })
      .def("col_t", [](const Block &b) { return b.col; })
      .def("eid_t", [](const Block &b) { return b.eid; })
      .def("ts_t", [](const Block &b) { return b.ts; })
      .def("dts_t", [](const Block &b) { return b.dts; })
      .def("nodes_t", [](const Block &b) { return b.nodes; })
      .def("uniE_t", [](const Block &b) { return b.uniE; })
      .def("invE_t", [](const Block &b) { return b.invE; })
      .def("cntE_t", [](const Block &b) { return b.cntE; })
      .def("rptr_t", [](const Block &b) { return b.rptr; });
  py::class_<Sampler>(m, "ParallelSampler")
      .def(py::init<py::object, py::object, py::object, py::object, int, int, int, std::vector<int>, bool, bool, int,
                    float, uint64_t>(),
           py::arg("indptr"), py::arg("indices"), py::arg("eid"), py::arg("ts"), py::arg("num_thread_per_worker"),
           py::arg("num_workers"), py::arg("num_layers"), py::arg("num_neighbors"), py::arg("recent"),
           py::arg("prop_time"), py::arg("num_history"), py::arg("window_duration"), py::arg("seed") = 0)
      .def("sample", &Sampler::sample, py::arg("root_nodes"), py::arg("root_ts"),
           py::arg("csrFlag") = std::vector<int>())
      .def("sample_device", &Sampler::sample_device)
      .def("update_pointers", &Sampler::update_pointers)
      .def("sample_shard", &Sampler::sample_shard)
      .def("reset", &Sampler::reset)
      .def("get_ret", &Sampler::get_ret)
      .def("dims", &Sampler::dims)
      .def("block_views", &Sampler::block_views)
      .def("dedup", &Sampler::dedup)
      .def("set_call_index", &Sampler::set_call_index)
      .def("configOMP", [](Sampler &, py::args, py::kwargs) {})
      .def("clear_cpu_affinity", [](Sampler &, py::args, py::kwargs) {})
      .def("check_bind", [](Sampler &, int) {}, py::arg("see_num"));
}
