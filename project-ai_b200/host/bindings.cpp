// Python bindings of the host runtime (module projectai_b200._paihost).
#include <pybind11/functional.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "runtime.h"

namespace py = pybind11;
using namespace paihost;

namespace {

Dims to_dims(const py::sequence& s) {
  Dims d;
  for (auto x : s) d.push_back(x.cast<int>());
  return d;
}

Tensor from_numpy(NativeBackend& be, py::array_t<float, py::array::c_style | py::array::forcecast> a, py::object shape) {
  Dims d;
  if (shape.is_none()) {
    for (py::ssize_t i = 0; i < a.ndim(); i++) d.push_back((int)a.shape(i));
  } else {
    d = to_dims(shape.cast<py::sequence>());
  }
  return be.from_host(a.data(), (int64_t)a.size(), d);
}

py::array_t<float> to_numpy(NativeBackend& be, const Tensor& t) {
  std::vector<py::ssize_t> shape(t->shape.begin(), t->shape.end());
  py::array_t<float> out(shape);
  {
    py::gil_scoped_release nogil;
    be.to_host(t, out.mutable_data(), t->numel());
  }
  return out;
}

// A model together with the context objects its modules hold references to (ParameterContext).
struct PyModel {
  std::shared_ptr<NativeBackend> be;
  std::unique_ptr<Autograd> ag;
  std::unique_ptr<PcgRng> rng;
  std::unique_ptr<LlamaModel> model;
};

struct PyTrainer {
  std::shared_ptr<PyModel> model;
  std::unique_ptr<Trainer> trainer;
};

std::vector<float> to_floats(const py::handle& h) {
  auto a = py::array_t<float, py::array::c_style | py::array::forcecast>::ensure(h);
  if (!a) throw ArgumentError("expected an array of token ids");
  return std::vector<float>(a.data(), a.data() + a.size());
}

}  // namespace

PYBIND11_MODULE(_paihost, m) {
  m.doc() = "C++ host runtime above the projectai_cuda C ABI (tensor views, autograd, Llama, AdamW, trainer, decode)";

  auto backend_error = py::register_exception<BackendError>(m, "BackendError", PyExc_RuntimeError);
  auto argument_error = py::register_exception<ArgumentError>(m, "ArgumentError", backend_error.ptr());
  py::register_exception<OutOfRangeError>(m, "OutOfRangeError", argument_error.ptr());
  py::register_exception<InvalidOperationError>(m, "InvalidOperationError", backend_error.ptr());
  py::register_exception<OutOfMemoryError>(m, "OutOfMemoryError", PyExc_MemoryError);
  py::register_exception<DeviceTimeoutError>(m, "DeviceTimeoutError", PyExc_TimeoutError);
  py::register_exception<FileIOError>(m, "FileIOError", PyExc_OSError);
  py::register_exception<InvalidDataError>(m, "InvalidDataError", PyExc_ValueError);

  py::class_<TensorImpl, Tensor>(m, "Tensor")
      .def_property_readonly("shape", [](const Tensor& t) { return py::tuple(py::cast(t->shape)); })
      .def_property_readonly("strides", [](const Tensor& t) { return py::tuple(py::cast(t->strides)); })
      .def_property_readonly("offset", [](const Tensor& t) { return t->offset; })
      .def_property("requires_grad", [](const Tensor& t) { return t->requires_grad; },
                    [](const Tensor& t, bool v) { t->requires_grad = v; })
      .def_property("grad", [](const Tensor& t) { return t->grad; }, [](const Tensor& t, Tensor g) { t->grad = g; })
      .def_property_readonly("grad_fn", [](const Tensor& t) { return t->grad_fn ? py::cast(t->grad_fn->op) : py::none(); })
      .def("numel", [](const Tensor& t) { return t->numel(); })
      .def("is_contiguous", [](const Tensor& t) { return t->is_contiguous(); })
      .def("backward", [](const Tensor& t, const Tensor& seed) { if (seed) t->backward(seed); else t->backward(); },
           py::arg("seed") = Tensor())
      .def("reshape", [](const Tensor& t, const py::sequence& d) { return t->reshape(to_dims(d)); })
      .def("transpose", [](const Tensor& t, int a, int b) { return t->transpose(a, b); })
      .def("permute", [](const Tensor& t, std::vector<int> p) { return t->permute(p); })
      .def("slice", [](const Tensor& t, int axis, int start, int length) { return t->slice(axis, start, length); })
      .def("broadcast_to", [](const Tensor& t, const py::sequence& d) { return t->broadcast_to(to_dims(d)); })
      .def("__repr__", [](const Tensor& t) { return "Tensor(shape=" + dims_str(t->shape) + ")"; });

  py::class_<NativeBackend, std::shared_ptr<NativeBackend>>(m, "Backend")
      .def(py::init<const std::string&, const std::string&, int>(), py::arg("library"), py::arg("prefix") = "pai_",
           py::arg("device") = 0)
      .def_property_readonly("name", &NativeBackend::name)
      .def_property_readonly("has_fused", &NativeBackend::has_fused)
      .def_readwrite("use_fused", &NativeBackend::use_fused)
      .def_readonly("dp_world", &NativeBackend::dp_world)
      .def_readonly("dp_rank", &NativeBackend::dp_rank)
      .def("from_host", [](NativeBackend& be, py::array a, py::object shape) { return from_numpy(be, a, shape); },
           py::arg("data"), py::arg("shape") = py::none())
      .def("to_host", [](NativeBackend& be, const Tensor& t) { return to_numpy(be, t); })
      .def("allocate", [](NativeBackend& be, const py::sequence& d) { return be.allocate(to_dims(d)); })
      .def("copy", &NativeBackend::copy)
      .def("add", &NativeBackend::add).def("sub", &NativeBackend::sub).def("mul", &NativeBackend::mul)
      .def("div", &NativeBackend::div).def("add_scalar", &NativeBackend::add_scalar)
      .def("mul_scalar", &NativeBackend::mul_scalar).def("sqrt", &NativeBackend::sqrt)
      .def("sigmoid", &NativeBackend::sigmoid).def("silu", &NativeBackend::silu)
      .def("matmul", &NativeBackend::matmul, py::arg("a"), py::arg("b"), py::arg("transpose_b") = false)
      .def("sum", &NativeBackend::sum, py::arg("x"), py::arg("axis"), py::arg("keep_dims") = false)
      .def("mean", &NativeBackend::mean, py::arg("x"), py::arg("axis"), py::arg("keep_dims") = false)
      .def("max", &NativeBackend::max, py::arg("x"), py::arg("axis"), py::arg("keep_dims") = false)
      .def("softmax", &NativeBackend::softmax).def("rms_norm", &NativeBackend::rms_norm)
      .def("rotary", &NativeBackend::rotary).def("gather", &NativeBackend::gather)
      .def("scatter_add_rows", &NativeBackend::scatter_add_rows).def("cross_entropy", &NativeBackend::cross_entropy)
      .def("cross_entropy_grad", &NativeBackend::cross_entropy_grad).def("cat", &NativeBackend::cat)
      .def("begin_scope", &NativeBackend::begin_scope).def("end_scope", &NativeBackend::end_scope)
      .def("keep_alive", &NativeBackend::keep_alive).def("release", &NativeBackend::release)
      .def("sync", &NativeBackend::sync, py::call_guard<py::gil_scoped_release>())
      .def("memory_stats", [](NativeBackend& be) {
        int64_t a = 0, b = 0, c = 0;
        be.memory_stats(&a, &b, &c);
        return py::make_tuple(a, b, c);
      })
      .def("reset_peak", &NativeBackend::reset_peak)
      .def("timer_start", &NativeBackend::timer_start)
      .def("timer_stop", &NativeBackend::timer_stop, py::call_guard<py::gil_scoped_release>())
      .def("launch_count", &NativeBackend::launch_count)
      .def("kernel_timing", &NativeBackend::kernel_timing)
      .def("kernel_stats", [](NativeBackend& be, const std::string& fam) {
        int64_t n = 0;
        double ms = 0, work = 0;
        be.kernel_stats(fam, &n, &ms, &work);
        return py::make_tuple(n, ms, work);
      })
      .def("check_device_error", &NativeBackend::check_device_error)
      .def_property_readonly("has_graphs", &NativeBackend::has_graphs)
      .def_property_readonly("has_decode_fusions", &NativeBackend::has_decode_fusions)
      .def("write", [](NativeBackend& be, const Tensor& dst, py::array_t<float, py::array::c_style | py::array::forcecast> a) {
        be.write(dst, a.data(), (int64_t)a.size());
      })
      .def("gather_dev", &NativeBackend::gather_dev)
      .def("save_checkpoint", &NativeBackend::save_checkpoint, py::arg("path"), py::arg("step"), py::arg("tensors"),
           py::arg("metadata") = "")
      .def("wait_checkpoint", &NativeBackend::wait_checkpoint, py::call_guard<py::gil_scoped_release>())
      .def("load_checkpoint", [](NativeBackend& be, const std::string& path, bool header_only) {
        auto r = be.load_checkpoint(path, header_only);
        return py::make_tuple(r.step, r.metadata, r.tensors);
      }, py::arg("path"), py::arg("header_only") = false)
      .def("dataset_open", &NativeBackend::dataset_open)
      .def("dataset_batch", &NativeBackend::dataset_batch)
      .def("dataset_close", &NativeBackend::dataset_close)
      .def("rotary_at", &NativeBackend::rotary_at)
      .def("kv_append", &NativeBackend::kv_append)
      .def("sdpa_decode", &NativeBackend::sdpa_decode)
      .def_property_readonly("has_argmax_rows", &NativeBackend::has_argmax_rows)
      .def("argmax_rows", &NativeBackend::argmax_rows)
      .def("linear_fused", &NativeBackend::linear_fused, py::arg("x"), py::arg("weights"), py::arg("mode"),
           py::arg("residual") = nullptr, py::arg("norm_weight") = nullptr, py::arg("eps") = 0.0f)
      .def("rope_append", &NativeBackend::rope_append)
      .def("attn_decode_step", &NativeBackend::attn_decode_step)
      .def("sdpa_fwd", [](NativeBackend& be, const Tensor& q, const Tensor& k, const Tensor& v, float scale, bool causal,
                          int pos) { return be.sdpa_fwd(q, k, v, scale, causal, pos); })
      .def("sdpa_bwd", &NativeBackend::sdpa_bwd)
      // CUDA graph capture of the ops issued between begin and end; the handle is an opaque integer
      .def("graph_begin", &NativeBackend::graph_begin)
      .def("graph_end", [](NativeBackend& be) { return reinterpret_cast<uintptr_t>(be.graph_end()); })
      .def("graph_launch", [](NativeBackend& be, uintptr_t g) { be.graph_launch(reinterpret_cast<pai_graph*>(g)); })
      .def("graph_destroy", [](NativeBackend& be, uintptr_t g) { be.graph_destroy(reinterpret_cast<pai_graph*>(g)); })
      .def("nccl_unique_id", [](NativeBackend& be) {
        uint8_t id[128];
        be.nccl_unique_id(id);
        return py::bytes(reinterpret_cast<char*>(id), 128);
      })
      .def("dp_stats", [](NativeBackend& be) { return be.dp_stats(); })
      .def("nccl_abort", &NativeBackend::nccl_abort)
      .def("nccl_init", [](NativeBackend& be, py::bytes id, int rank, int world, int timeout_ms) {
        std::string s = id;
        if (s.size() != 128) throw ArgumentError("NCCL unique id must be 128 bytes");
        py::gil_scoped_release nogil;
        be.nccl_init(reinterpret_cast<const uint8_t*>(s.data()), rank, world, timeout_ms);
      });

  struct NoGradCtx { std::unique_ptr<GradMode::Guard> g; bool disabled; };
  py::class_<NoGradCtx>(m, "GradModeScope")
      .def("__enter__", [](NoGradCtx& c) { c.g = std::make_unique<GradMode::Guard>(c.disabled); })
      .def("__exit__", [](NoGradCtx& c, py::object, py::object, py::object) { c.g.reset(); });
  m.def("no_grad", []() { return NoGradCtx{nullptr, true}; });
  m.def("enable_grad", []() { return NoGradCtx{nullptr, false}; });
  m.def("grad_enabled", &GradMode::enabled);

  py::class_<Autograd>(m, "Autograd")
      .def(py::init([](std::shared_ptr<NativeBackend> be) { return new Autograd(be.get()); }), py::keep_alive<1, 2>())
      .def("add", &Autograd::add).def("sub", &Autograd::sub).def("mul", &Autograd::mul)
      .def("matmul", &Autograd::matmul, py::arg("a"), py::arg("b"), py::arg("transpose_b") = false)
      .def("contiguous", &Autograd::contiguous).def("sum_all", &Autograd::sum_all).def("mean", &Autograd::mean)
      .def("embedding", &Autograd::embedding).def("cross_entropy", &Autograd::cross_entropy)
      .def("softmax", &Autograd::softmax).def("silu", &Autograd::silu).def("rms_norm", &Autograd::rms_norm)
      .def("rotary", static_cast<Tensor (Autograd::*)(const Tensor&, const Tensor&, const Tensor&)>(&Autograd::rotary))
      .def("transpose", &Autograd::transpose).def("permute", &Autograd::permute)
      .def("reshape", [](Autograd& ag, const Tensor& x, const py::sequence& d) { return ag.reshape(x, to_dims(d)); })
      .def("slice", &Autograd::slice)
      .def("broadcast_to", [](Autograd& ag, const Tensor& x, const py::sequence& d) { return ag.broadcast_to(x, to_dims(d)); })
      .def("silu_mul", &Autograd::silu_mul).def("attention", &Autograd::attention)
      .def("checkpoint", [](Autograd& ag, py::function seg, const Tensor& input, std::vector<Tensor> params) {
        std::function<Tensor(const Tensor&)> f = [seg](const Tensor& x) {
          py::gil_scoped_acquire gil;
          return seg(x).cast<Tensor>();
        };
        return ag.checkpoint(f, input, params);
      });

  py::class_<PcgRng>(m, "PcgRng")
      .def(py::init<uint64_t, uint64_t>(), py::arg("seed"), py::arg("stream") = 0xDA3E39CB94B95BDBull)
      .def("next_u32", &PcgRng::next_u32).def("next_float", &PcgRng::next_float)
      .def("next_gaussian", &PcgRng::next_gaussian);

  py::class_<ModelConfig>(m, "ModelConfig")
      .def(py::init([](int vocab, int dim, int layers, int heads, int kv_heads, int ffn, int max_seq, float theta, float eps) {
             ModelConfig c;
             c.vocab_size = vocab; c.embedding_dim = dim; c.layer_count = layers; c.head_count = heads;
             c.kv_head_count = kv_heads; c.ffn_hidden = ffn; c.max_sequence_length = max_seq;
             c.rope_theta = theta; c.norm_eps = eps;
             c.validate();
             return c;
           }),
           py::arg("vocab_size"), py::arg("embedding_dim"), py::arg("layer_count"), py::arg("head_count"),
           py::arg("kv_head_count"), py::arg("ffn_hidden"), py::arg("max_sequence_length") = 4096,
           py::arg("rope_theta") = 10000.0f, py::arg("norm_eps") = 1e-5f)
      .def_readonly("vocab_size", &ModelConfig::vocab_size).def_readonly("embedding_dim", &ModelConfig::embedding_dim)
      .def_readonly("layer_count", &ModelConfig::layer_count).def_readonly("head_count", &ModelConfig::head_count)
      .def_readonly("kv_head_count", &ModelConfig::kv_head_count).def_readonly("ffn_hidden", &ModelConfig::ffn_hidden)
      .def_readonly("max_sequence_length", &ModelConfig::max_sequence_length)
      .def_readonly("rope_theta", &ModelConfig::rope_theta).def_readonly("norm_eps", &ModelConfig::norm_eps)
      .def_property_readonly("head_dim", &ModelConfig::head_dim);

  py::class_<PyModel, std::shared_ptr<PyModel>>(m, "LlamaModel")
      .def(py::init([](std::shared_ptr<NativeBackend> be, const ModelConfig& cfg, uint64_t seed, const std::string& init,
                       bool skip_init) {
             auto pm = std::make_shared<PyModel>();
             pm->be = be;
             pm->ag = std::make_unique<Autograd>(be.get());
             pm->rng = std::make_unique<PcgRng>(seed);
             ParameterContext ctx{be.get(), pm->ag.get(), pm->rng.get(), skip_init, std::nullopt};
             if (init == "normal0.02") ctx.override_init = Initializer{InitKind::Normal, 0.0f, 0.02f};
             else if (init != "reference") throw ArgumentError("init must be 'reference' or 'normal0.02'");
             py::gil_scoped_release nogil;
             pm->model = std::make_unique<LlamaModel>(ctx, cfg);
             return pm;
           }),
           py::arg("backend"), py::arg("config"), py::arg("seed") = 0, py::arg("init") = "reference",
           py::arg("skip_init") = false)
      .def("forward", [](PyModel& pm, const Tensor& ids, KvCache* cache) {
        py::gil_scoped_release nogil;
        ForwardContext ctx;
        ctx.cache = cache;
        return pm.model->forward(ids, ctx);
      }, py::arg("ids"), py::arg("cache") = nullptr)
      .def("attention", [](PyModel& pm, int layer, const Tensor& x) {
        if (layer < 0 || layer >= (int)pm.model->blocks.size()) throw OutOfRangeError("layer out of range");
        return pm.model->blocks[(size_t)layer]->attn->forward(x, ForwardContext{});
      })
      .def_property("gradient_checkpointing", [](PyModel& pm) { return pm.model->gradient_checkpointing; },
                    [](PyModel& pm, bool v) { pm.model->gradient_checkpointing = v; })
      .def("named_parameters", [](PyModel& pm) { return pm.model->named_parameters(); })
      .def("parameters", [](PyModel& pm) { return pm.model->parameters(); })
      .def_property_readonly("autograd", [](PyModel& pm) { return pm.ag.get(); }, py::return_value_policy::reference_internal)
      .def_property_readonly("config", [](PyModel& pm) { return pm.model->cfg; });

  py::class_<KvCache>(m, "KvCache")
      .def(py::init([](std::shared_ptr<NativeBackend> be, std::shared_ptr<PyModel> pm, int max_batch, int max_seq) {
             return new KvCache(be.get(), pm->model->cfg, max_batch, max_seq);
           }),
           py::arg("backend"), py::arg("model"), py::arg("max_batch") = 1, py::arg("max_sequence_length") = 4096,
           py::keep_alive<1, 2>())
      .def("length", &KvCache::length)
      .def("reset", &KvCache::reset);

  py::class_<GraphDecoder>(m, "GraphDecoder")
      .def(py::init([](std::shared_ptr<NativeBackend> be, std::shared_ptr<PyModel> pm, KvCache& cache, int batch) {
             return new GraphDecoder(be.get(), pm->model.get(), &cache, batch);
           }),
           py::arg("backend"), py::arg("model"), py::arg("cache"), py::arg("batch") = 1, py::keep_alive<1, 2>(),
           py::keep_alive<1, 3>(), py::keep_alive<1, 4>())
      .def("step", [](GraphDecoder& g, std::vector<int> ids) {
        GradMode::Guard nograd(true);
        return g.step(ids);
      })
      .def_property_readonly("captured", &GraphDecoder::captured)
      .def_readwrite("fused", &GraphDecoder::fused);
  m.def("has_graphs", [](std::shared_ptr<NativeBackend> be) { return be->has_graphs(); });

  m.def("cross_entropy_loss", [](Autograd& ag, const Tensor& logits, const Tensor& targets, int ignore) {
    return cross_entropy_loss(ag, logits, targets, ignore);
  }, py::arg("ag"), py::arg("logits"), py::arg("targets"), py::arg("ignore_index") = -100);

  py::class_<AdamW>(m, "AdamW")
      .def(py::init([](std::vector<Tensor> params, std::shared_ptr<NativeBackend> be, float lr, float b1, float b2, float eps,
                       float wd) { return new AdamW(params, be.get(), lr, b1, b2, eps, wd); }),
           py::arg("params"), py::arg("backend"), py::arg("lr") = 1e-3f, py::arg("beta1") = 0.9f, py::arg("beta2") = 0.999f,
           py::arg("eps") = 1e-8f, py::arg("weight_decay") = 0.01f, py::keep_alive<1, 3>())
      .def("step", &AdamW::step).def("zero_grad", &AdamW::zero_grad)
      .def_readwrite("lr", &AdamW::lr).def_readwrite("grad_scale", &AdamW::grad_scale)
      .def_readonly("step_count", &AdamW::step_count)
      .def("set_schedule", [](AdamW& o, std::function<float(int)> f) { o.schedule = f; })
      .def("state_t", [](AdamW& o, const Tensor& p) {
        auto it = o.state.find(p.get());
        return it == o.state.end() ? 0 : it->second.t;
      });

  py::class_<TrainingConfig>(m, "TrainingConfig")
      .def(py::init([](int batch, int seq, float lr, float wd, int max_steps, int accum, bool ckpt, int warmup, uint64_t seed,
                       int ckpt_every, const std::string& ckpt_dir) {
             TrainingConfig c;
             c.batch_size = batch; c.sequence_length = seq; c.learning_rate = lr; c.weight_decay = wd;
             c.max_steps = max_steps; c.grad_accum = accum; c.gradient_checkpointing = ckpt; c.warmup_steps = warmup;
             c.seed = seed; c.checkpoint_every_steps = ckpt_every; c.checkpoint_directory = ckpt_dir;
             return c;
           }),
           py::arg("batch_size") = 8, py::arg("sequence_length") = 512, py::arg("learning_rate") = 3e-4f,
           py::arg("weight_decay") = 0.01f, py::arg("max_steps") = 1000, py::arg("grad_accum") = 1,
           py::arg("gradient_checkpointing") = false, py::arg("warmup_steps") = 100, py::arg("seed") = 0,
           py::arg("checkpoint_every_steps") = 0, py::arg("checkpoint_directory") = "checkpoints");

  py::class_<PyTrainer>(m, "Trainer")
      .def(py::init([](std::shared_ptr<NativeBackend> be, std::shared_ptr<PyModel> model, const TrainingConfig& cfg,
                       float beta1, float beta2) {
             auto* t = new PyTrainer();
             t->model = model;
             t->trainer = std::make_unique<Trainer>(be.get(), model->model.get(), cfg, beta1, beta2);
             return t;
           }),
           py::arg("backend"), py::arg("model"), py::arg("config"), py::arg("beta1") = 0.9f, py::arg("beta2") = 0.999f,
           py::keep_alive<1, 2>())
      .def("step", [](PyTrainer& t, py::list inputs, py::list targets) {
        std::vector<std::vector<float>> in, tg;
        for (auto h : inputs) in.push_back(to_floats(h));
        for (auto h : targets) tg.push_back(to_floats(h));
        py::gil_scoped_release nogil;
        return t.trainer->step(in, tg);
      })
      .def("step_tensors", [](PyTrainer& t, std::vector<Tensor> inputs, std::vector<Tensor> targets) {
        py::gil_scoped_release nogil;
        return t.trainer->step_tensors(inputs, targets);
      })
      .def("save_checkpoint", [](PyTrainer& t, const std::string& path, int step, const std::string& metadata) {
        py::gil_scoped_release nogil;
        t.trainer->save_checkpoint(path, step, metadata);
      }, py::arg("path"), py::arg("step"), py::arg("metadata") = "")
      .def("wait_checkpoint", [](PyTrainer& t) {
        py::gil_scoped_release nogil;
        t.trainer->wait_checkpoint();
      })
      .def("restore", [](PyTrainer& t, const std::string& path) {
        py::gil_scoped_release nogil;
        return t.trainer->restore(path);
      })
      // Trainer.Train over host sequences (lists of int ids) or, with packed_blocks > 0, the backend's open packed
      // dataset; on_step(step, loss) is called with the GIL held. Returns the TrainingReport as a dict.
      .def("train", [](PyTrainer& t, py::object sequences, int64_t packed_blocks, py::object on_step) {
        std::unique_ptr<SequenceSource> src;
        if (packed_blocks > 0) {
          auto p = std::make_unique<PackedSequences>();
          p->blocks = packed_blocks;
          src = std::move(p);
        } else {
          auto h = std::make_unique<HostSequences>();
          if (!sequences.is_none())
            for (auto seq : sequences) h->seqs.push_back(seq.cast<std::vector<int32_t>>());
          src = std::move(h);
        }
        std::function<void(int, float)> cb;
        if (!on_step.is_none())
          cb = [on_step](int step, float loss) {
            py::gil_scoped_acquire gil;
            on_step(step, loss);
          };
        TrainingReport r;
        {
          py::gil_scoped_release nogil;
          r = t.trainer->train(*src, cb);
        }
        py::dict d;
        d["step_losses"] = r.step_losses;
        d["final_step"] = r.final_step;
        d["first_loss"] = r.step_losses.empty() ? NAN : r.step_losses.front();
        d["last_loss"] = r.step_losses.empty() ? NAN : r.step_losses.back();
        return d;
      }, py::arg("sequences") = py::none(), py::arg("packed_blocks") = 0, py::arg("on_step") = py::none())
      // (name, tensor) pairs of the checkpointed state with full-size moments; collective under ZeRO-1
      .def("state_items", [](PyTrainer& t) {
        py::gil_scoped_release nogil;
        return t.trainer->state_items();
      })
      .def("apply_state", [](PyTrainer& t, const std::vector<std::pair<std::string, Tensor>>& items, int step) {
        py::gil_scoped_release nogil;
        t.trainer->apply_state(items, step);
      }, py::arg("items"), py::arg("step"))
      .def_property_readonly("optimizer", [](PyTrainer& t) { return t.trainer->optimizer.get(); },
                             py::return_value_policy::reference_internal)
      .def("set_constant_lr", [](PyTrainer& t, float lr) {
        t.trainer->optimizer->schedule = [lr](int) { return lr; };
      })
      .def_property("world", [](PyTrainer& t) { return t.trainer->world; },
                    [](PyTrainer& t, int w) { t.trainer->world = w; })
      // fn(list[Tensor]) must sum each tensor in place across ranks (called with the GIL held).
      .def("set_allreduce", [](PyTrainer& t, py::function fn) {
        t.trainer->allreduce = [fn](const std::vector<Tensor>& grads) {
          py::gil_scoped_acquire gil;
          fn(grads);
        };
        t.trainer->allreduce_wait = [] {};
      })
      // ZeRO-1 (sharded AdamW state); with CPU collectives substituted for the backend's NCCL exchanges in tests
      .def_property("zero1", [](PyTrainer& t) { return t.trainer->zero1; },
                    [](PyTrainer& t, bool v) { t.trainer->zero1 = v; })
      .def_property("rank", [](PyTrainer& t) { return t.trainer->rank; },
                    [](PyTrainer& t, int v) { t.trainer->rank = v; })
      .def("set_shard_exchange", [](PyTrainer& t, py::function reduce_scatter, py::function allgather) {
        t.trainer->reduce_scatter = [reduce_scatter](const std::vector<Tensor>& g) {
          py::gil_scoped_acquire gil;
          reduce_scatter(g);
        };
        t.trainer->allgather = [allgather](const std::vector<Tensor>& p) {
          py::gil_scoped_acquire gil;
          allgather(p);
        };
      })
      .def("moment_elements", [](PyTrainer& t) {
        int64_t n = 0;
        for (auto& kv : t.trainer->optimizer->state)
          if (kv.second.m) n += kv.second.m->numel() + kv.second.v->numel();
        return n;
      });

  m.def("apply_weights", [](std::shared_ptr<NativeBackend> be, std::shared_ptr<PyModel> model,
                            const std::vector<std::pair<std::string, Tensor>>& items) {
    py::gil_scoped_release nogil;
    apply_weights(be.get(), model->model.get(), items);
  }, py::arg("backend"), py::arg("model"), py::arg("items"));

  py::class_<TopKTopPSampler>(m, "TopKTopPSampler")
      .def(py::init<uint64_t, float, int, float>(), py::arg("seed"), py::arg("temperature") = 1.0f, py::arg("top_k") = 0,
           py::arg("top_p") = 1.0f)
      .def("sample", [](TopKTopPSampler& s, py::array_t<float, py::array::c_style | py::array::forcecast> a) {
        return s.sample(a.data(), (int)a.size());
      })
      .def("sample_rows", [](TopKTopPSampler& s, py::array_t<float, py::array::c_style | py::array::forcecast> a) {
        if (a.ndim() != 2) throw ArgumentError("sample_rows expects [rows, vocab] logits");
        std::vector<int> out((size_t)a.shape(0));
        s.sample_rows(a.data(), (int)a.shape(0), (int)a.shape(1), out.data());
        return out;
      });
  m.def("argmax", [](py::array_t<float, py::array::c_style | py::array::forcecast> a) { return argmax(a.data(), (int)a.size()); });

  m.def("generate", [](std::shared_ptr<NativeBackend> be, std::shared_ptr<PyModel> model, std::vector<int> prompt, int max_tokens,
                       TopKTopPSampler* sampler, int batch) {
    GenerateResult r;
    {
      py::gil_scoped_release nogil;
      r = generate(be.get(), model->model.get(), prompt, max_tokens, sampler, batch);
    }
    py::dict d;
    d["tokens"] = r.tokens;
    d["prefill_seconds"] = r.prefill_seconds;
    d["decode_seconds"] = r.decode_seconds;
    d["graph"] = r.graph;
    return d;
  }, py::arg("backend"), py::arg("model"), py::arg("prompt"), py::arg("max_tokens"), py::arg("sampler") = nullptr,
     py::arg("batch") = 1);
}
