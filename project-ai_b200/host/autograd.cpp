// The differentiable op layer: a restatement of ProjectAI.Core/Autograd.cs (rule by rule, same op order) plus one node
// per fused extension. GradMode.cs: thread-local on/off switch.
#include <cmath>

#include "runtime.h"

namespace paihost {

static thread_local bool t_grad_disabled = false;

bool GradMode::enabled() { return !t_grad_disabled; }
GradMode::Guard::Guard(bool disabled) : previous(t_grad_disabled) { t_grad_disabled = disabled; }
GradMode::Guard::~Guard() { t_grad_disabled = previous; }

// Autograd.Record (Autograd.cs:308-317).
Tensor Autograd::record(const Tensor& y, const std::string& op, std::vector<Tensor> inputs,
                        std::function<std::vector<Tensor>(const Tensor&)> backward) {
  y->backend = be;
  bool any = false;
  for (const auto& in : inputs) any = any || in->requires_grad;
  if (GradMode::enabled() && any) {
    y->requires_grad = true;
    auto node = std::make_shared<GradNode>();
    node->op = op;
    node->inputs = std::move(inputs);
    node->backward = std::move(backward);
    y->grad_fn = node;
  }
  return y;
}

// ReduceGradToShape (Autograd.cs:320-333).
Tensor Autograd::reduce_grad_to_shape(const Tensor& grad, const Dims& target) {
  if (grad->shape == target) return grad;
  Tensor g = grad;
  int lead = grad->rank() - (int)target.size();
  for (int i = 0; i < lead; i++) g = be->sum(g, 0);
  for (int axis = 0; axis < (int)target.size(); axis++)
    if (target[(size_t)axis] == 1 && g->shape[(size_t)axis] != 1) g = be->sum(g, axis, true);
  return g;
}

// ToScalar (Autograd.cs:335-340). A value the host already knows needs no device read-back.
float Autograd::to_scalar(const Tensor& t) {
  float v = 0.0f;
  be->to_host(t, &v, 1);
  return v;
}

Tensor Autograd::add(const Tensor& a, const Tensor& b) {
  Tensor y = be->add(a, b);
  Dims sa = a->shape, sb = b->shape;
  return record(y, "add", {a, b}, [this, sa, sb](const Tensor& g) {
    return std::vector<Tensor>{reduce_grad_to_shape(g, sa), reduce_grad_to_shape(g, sb)};
  });
}

Tensor Autograd::sub(const Tensor& a, const Tensor& b) {
  Tensor y = be->sub(a, b);
  Dims sa = a->shape, sb = b->shape;
  return record(y, "sub", {a, b}, [this, sa, sb](const Tensor& g) {
    Tensor gb = reduce_grad_to_shape(be->mul_scalar(g, -1.0f), sb);
    return std::vector<Tensor>{reduce_grad_to_shape(g, sa), gb};
  });
}

Tensor Autograd::mul(const Tensor& a, const Tensor& b) {
  Tensor y = be->mul(a, b);
  return record(y, "mul", {a, b}, [this, a, b](const Tensor& g) {
    Tensor ga = reduce_grad_to_shape(be->mul(g, b), a->shape);
    Tensor gb = reduce_grad_to_shape(be->mul(g, a), b->shape);
    return std::vector<Tensor>{ga, gb};
  });
}

static Tensor last_t(const Tensor& t) { return t->transpose(t->rank() - 2, t->rank() - 1); }

// MatMul (Autograd.cs:54-73).
Tensor Autograd::matmul(const Tensor& a, const Tensor& b, bool tb) {
  if (a->rank() < 2 || b->rank() < 2)
    throw ArgumentError("MatMul requires rank >= 2 operands; got " + dims_str(a->shape) + " and " + dims_str(b->shape) + ".");
  Tensor y = be->matmul(a, b, tb);
  if (!tb)
    return record(y, "matmul", {a, b}, [this, a, b](const Tensor& g) {
      Tensor ga = reduce_grad_to_shape(be->matmul(g, b, true), a->shape);  // g · bᵀ
      Tensor gb = reduce_grad_to_shape(be->matmul(last_t(a), g), b->shape);  // aᵀ · g
      return std::vector<Tensor>{ga, gb};
    });
  return record(y, "matmul_tb", {a, b}, [this, a, b](const Tensor& g) {
    Tensor ga = reduce_grad_to_shape(be->matmul(g, b), a->shape);          // g · b
    Tensor gb = reduce_grad_to_shape(be->matmul(last_t(g), a), b->shape);  // gᵀ · a
    return std::vector<Tensor>{ga, gb};
  });
}

// Contiguous (Autograd.cs:83-89).
Tensor Autograd::contiguous(const Tensor& x) {
  if (x->is_contiguous() && x->offset == 0) return x;
  Tensor dst = be->allocate(x->shape);
  be->copy(x, dst);
  return record(dst, "contiguous", {x}, [](const Tensor& g) { return std::vector<Tensor>{g}; });
}

// SumAll (Autograd.cs:92-98).
Tensor Autograd::sum_all(const Tensor& x) {
  Tensor y = x;
  for (int axis = x->rank() - 1; axis >= 0; axis--) y = be->sum(y, axis);
  Dims sx = x->shape;
  return record(y, "sum_all", {x}, [this, sx](const Tensor& g) {
    return std::vector<Tensor>{be->add_scalar(be->allocate(sx), to_scalar(g))};
  });
}

// Mean (Autograd.cs:160-171).
Tensor Autograd::mean(const Tensor& x) {
  int64_t count = x->numel();
  Tensor y = x;
  for (int axis = x->rank() - 1; axis >= 0; axis--) y = be->mean(y, axis);
  Dims sx = x->shape;
  return record(y, "mean", {x}, [this, sx, count](const Tensor& g) {
    float scaled = to_scalar(g) / (float)count;
    return std::vector<Tensor>{be->add_scalar(be->allocate(sx), scaled)};
  });
}

// DetachLeaf (Autograd.cs:151-158).
Tensor Autograd::detach_leaf(const Tensor& x) {
  Tensor copy = be->allocate(x->shape);
  be->copy(x, copy);
  copy->backend = be;
  copy->requires_grad = true;
  return copy;
}

// Checkpoint (Autograd.cs:120-147): a no-grad forward in its own scope, and a backward that recomputes the segment
// from a detached copy of the input inside a scope, runs the segment's backward from the upstream gradient, and keeps
// the input grad and the segment's parameter grads alive one level up. `on_grads_ready` runs once those parameter
// grads are final (the data-parallel bucket hook).
// The reference seeds that backward through the surrogate loss Σ(recomputed ⊙ upstream); the surrogate's gradient
// with respect to the recomputed output is 1·upstream, exactly upstream, so seeding the walk with upstream gives the
// same gradients bit for bit without computing the surrogate's (unused) value.
Tensor Autograd::checkpoint(const std::function<Tensor(const Tensor&)>& segment, const Tensor& input,
                            const std::vector<Tensor>& parameters, const std::function<void()>& on_grads_ready) {
  Tensor output;
  {
    GradMode::Guard nograd(true);
    be->begin_scope();
    try {
      output = segment(input);
      be->keep_alive(output);
    } catch (...) {
      be->end_scope();
      throw;
    }
    be->end_scope();
  }
  return record(output, "checkpoint", {input}, [this, segment, input, parameters, on_grads_ready](const Tensor& upstream) {
    be->begin_scope();
    Tensor input_grad;
    try {
      Tensor leaf = detach_leaf(input);
      Tensor recomputed;
      {
        GradMode::Guard enabled(false);
        recomputed = segment(leaf);
      }
      recomputed->backward(upstream);
      input_grad = leaf->grad ? leaf->grad : be->allocate(input->shape);
      be->keep_alive(input_grad);
      for (const auto& p : parameters)
        if (p->grad) be->keep_alive(p->grad);
    } catch (...) {
      be->end_scope();
      throw;
    }
    be->end_scope();
    if (on_grads_ready) on_grads_ready();
    return std::vector<Tensor>{input_grad};
  });
}

// Embedding (Autograd.cs:178-183).
Tensor Autograd::embedding(const Tensor& weight, const std::vector<int>& ids) {
  Tensor y = be->gather(weight, ids);
  int vocab = weight->shape[0];
  return record(y, "embedding", {weight}, [this, ids, vocab](const Tensor& g) {
    return std::vector<Tensor>{be->scatter_add_rows(g, ids, vocab)};
  });
}

// CrossEntropy (Autograd.cs:187-192). With the fused extension the gradient is produced by the same read of the
// logits as the loss, and the backward only scales it by the upstream scalar (skipped when that scalar is exactly 1).
Tensor Autograd::cross_entropy(const Tensor& logits, const std::vector<int>& targets, int ignore) {
  if (be->use_fused && be->has_fused() && GradMode::enabled() && logits->requires_grad) {
    auto lg = be->cross_entropy_fused(logits, targets, ignore, 1.0f);
    Tensor grad = lg.second;
    return record(lg.first, "cross_entropy", {logits}, [this, grad](const Tensor& g) {
      float s = to_scalar(g);
      return std::vector<Tensor>{s == 1.0f ? grad : be->mul_scalar(grad, s)};
    });
  }
  Tensor loss = be->cross_entropy(logits, targets, ignore);
  return record(loss, "cross_entropy", {logits}, [this, logits, targets, ignore](const Tensor& g) {
    return std::vector<Tensor>{be->mul_scalar(be->cross_entropy_grad(logits, targets, ignore), to_scalar(g))};
  });
}

// Softmax (Autograd.cs:197-205).
Tensor Autograd::softmax(const Tensor& x, int axis) {
  Tensor y = be->softmax(x, axis);
  std::weak_ptr<TensorImpl> wy = y;
  return record(y, "softmax", {x}, [this, wy, axis](const Tensor& g) {
    Tensor yy = wy.lock();
    Tensor dot = be->sum(be->mul(g, yy), axis, true);
    return std::vector<Tensor>{be->mul(yy, be->sub(g, dot))};
  });
}

// Silu (Autograd.cs:208-217).
Tensor Autograd::silu(const Tensor& x) {
  Tensor y = be->silu(x);
  std::weak_ptr<TensorImpl> wy = y;
  return record(y, "silu", {x}, [this, x, wy](const Tensor& g) {
    Tensor yy = wy.lock();
    Tensor s = be->sigmoid(x);
    Tensor derivative = be->sub(be->add(s, yy), be->mul(s, yy));
    return std::vector<Tensor>{be->mul(g, derivative)};
  });
}

// RmsNorm (Autograd.cs:223-244); the fused extension computes the same rule in one pass over x and g.
Tensor Autograd::rms_norm(const Tensor& x, const Tensor& w, float eps) {
  int last = x->rank() - 1;
  int d = x->shape[(size_t)last];
  Tensor y = be->rms_norm(x, w, eps);
  std::weak_ptr<TensorImpl> wy = y;
  return record(y, "rmsnorm", {x, w}, [this, x, w, wy, eps, last, d](const Tensor& g) {
    if (be->use_fused && be->has_fused()) {
      auto r = be->rms_norm_bwd(x, w, g, eps);
      return std::vector<Tensor>{r.first, r.second};
    }
    Tensor yy = wy.lock();
    Tensor mean_sq = be->mean(be->mul(x, x), last, true);
    Tensor denom = be->sqrt(be->add_scalar(mean_sq, eps));
    Tensor ones = be->add_scalar(be->allocate(denom->shape), 1.0f);
    Tensor inv = be->div(ones, denom);
    Tensor dot = be->sum(be->mul(g, yy), last, true);
    Tensor direct = be->mul(be->mul(g, w), inv);
    Tensor coef = be->mul_scalar(be->mul(inv, inv), 1.0f / (float)d);
    Tensor center = be->mul(be->mul(coef, x), dot);
    Tensor grad_x = be->sub(direct, center);
    Tensor grad_w = reduce_grad_to_shape(be->mul(g, be->mul(x, inv)), w->shape);
    return std::vector<Tensor>{grad_x, grad_w};
  });
}

// RotaryEmbedding (Autograd.cs:250-255).
Tensor Autograd::rotary(const Tensor& x, const Tensor& cos, const Tensor& sin) {
  return rotary(x, cos, sin, be->mul_scalar(sin, -1.0f));
}

Tensor Autograd::rotary(const Tensor& x, const Tensor& cos, const Tensor& sin, const Tensor& neg_sin) {
  Tensor y = be->rotary(x, cos, sin);
  return record(y, "rope", {x}, [this, cos, neg_sin](const Tensor& g) {
    return std::vector<Tensor>{be->rotary(g, cos, neg_sin)};
  });
}

// View ops (Autograd.cs:259-305).
Tensor Autograd::transpose(const Tensor& x, int a0, int a1) {
  Tensor y = x->transpose(a0, a1);
  return record(y, "transpose", {x}, [a0, a1](const Tensor& g) { return std::vector<Tensor>{g->transpose(a0, a1)}; });
}

Tensor Autograd::permute(const Tensor& x, const std::vector<int>& p) {
  std::vector<int> inv(p.size());
  for (size_t i = 0; i < p.size(); i++) inv[(size_t)p[i]] = (int)i;
  Tensor y = x->permute(p);
  return record(y, "permute", {x}, [inv](const Tensor& g) { return std::vector<Tensor>{g->permute(inv)}; });
}

Tensor Autograd::reshape(const Tensor& x, const Dims& d) {
  Dims original = x->shape;
  Tensor y = x->reshape(d);
  return record(y, "reshape", {x}, [this, original](const Tensor& g0) {
    Tensor g = g0;
    if (!(g->is_contiguous() && g->offset == 0)) {
      Tensor dense = be->allocate(g->shape);
      be->copy(g, dense);
      g = dense;
    }
    return std::vector<Tensor>{g->reshape(original)};
  });
}

Tensor Autograd::slice(const Tensor& x, int axis, int start, int length) {
  Dims shape = x->shape;
  Tensor y = x->slice(axis, start, length);
  return record(y, "slice", {x}, [this, shape, axis, start, length](const Tensor& g) {
    Tensor grad = be->allocate(shape);
    be->copy(g, grad->slice(axis, start, length));
    return std::vector<Tensor>{grad};
  });
}

Tensor Autograd::broadcast_to(const Tensor& x, const Dims& target) {
  Tensor y = x->broadcast_to(target);
  Dims sx = x->shape;
  return record(y, "broadcast", {x}, [this, sx](const Tensor& g) { return std::vector<Tensor>{reduce_grad_to_shape(g, sx)}; });
}

// SwiGLU gate silu(gate)·up as one node (the Silu rule Autograd.cs:208-217 composed with the Mul rule :39-47).
Tensor Autograd::silu_mul(const Tensor& gate, const Tensor& up) {
  if (!(be->use_fused && be->has_fused())) return mul(silu(gate), up);
  Tensor y = be->silu_mul(gate, up);
  return record(y, "silu_mul", {gate, up}, [this, gate, up](const Tensor& g) {
    auto r = be->silu_mul_bwd(gate, up, g);
    return std::vector<Tensor>{r.first, r.second};
  });
}

// Fused causal attention: q [B,H,S,D], k/v [B,KVH,L,D] -> [B,S,H,D]; one node whose backward is the fused
// attention backward (the MatMul, Softmax and GQA-sum rules of the composed chain).
Tensor Autograd::attention(const Tensor& q, const Tensor& k, const Tensor& v, float scale, int pos_offset) {
  auto ol = be->sdpa_fwd(q, k, v, scale, true, pos_offset);
  Tensor out = ol.first, lse = ol.second;
  std::weak_ptr<TensorImpl> wout = out;
  return record(out, "attention", {q, k, v}, [this, q, k, v, wout, lse, scale, pos_offset](const Tensor& g) {
    return be->sdpa_bwd(q, k, v, wout.lock(), lse, g, scale, true, pos_offset);
  });
}

}  // namespace paihost
