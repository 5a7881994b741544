// PcgRng and Init (ProjectAI.Core/Rng.cs, Init.cs), Module (Module.cs), the Llama modules (ProjectAI.Models/Modules.cs,
// Linear.cs, Embedding.cs, Loss.cs), the KV cache (Modules.cs:290-370) and the samplers (Sampling.cs).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <numeric>
#include <thread>

#include <pthread.h>
#include <unistd.h>

#include <new>

#include "runtime.h"

namespace paihost {

// ---------------------------------------------------------------- PcgRng (Rng.cs:25-60): PCG-XSH-RR 64/32, Box–Muller
PcgRng::PcgRng(uint64_t seed, uint64_t stream) {
  inc_ = (stream << 1) | 1ull;
  state_ = 0;
  next_u32();
  state_ += seed;
  next_u32();
}

uint32_t PcgRng::next_u32() {
  uint64_t old = state_;
  state_ = old * 6364136223846793005ull + inc_;
  uint32_t xorshifted = (uint32_t)(((old >> 18) ^ old) >> 27);
  uint32_t rot = (uint32_t)(old >> 59);
  return (xorshifted >> rot) | (xorshifted << ((0u - rot) & 31u));
}

float PcgRng::next_float() { return (float)(next_u32() >> 8) * (1.0f / (float)(1u << 24)); }

float PcgRng::next_gaussian() {
  if (has_spare_) {
    has_spare_ = false;
    return spare_;
  }
  float u1 = std::max(next_float(), 1e-7f);
  float u2 = next_float();
  float magnitude = sqrtf(-2.0f * logf(u1));
  const float two_pi = 2.0f * 3.14159265f;  // 2f * MathF.PI
  spare_ = magnitude * sinf(two_pi * u2);
  has_spare_ = true;
  return magnitude * cosf(two_pi * u2);
}

// ---------------------------------------------------------------- Init (Init.cs:22-75)
static std::pair<int64_t, int64_t> fans(const Dims& s) {
  if (s.size() <= 1) {
    int64_t n = s.empty() ? 1 : s[0];
    return {n, n};
  }
  int64_t fan_out = s[0], fan_in = 1;
  for (size_t i = 1; i < s.size(); i++) fan_in *= s[i];
  return {fan_in, fan_out};
}

static void fill_gaussian(const Tensor& target, NativeBackend& be, PcgRng& rng, float mean, float std) {
  std::vector<float> buf((size_t)target->numel());
  for (auto& x : buf) x = mean + std * rng.next_gaussian();
  be.copy(be.from_host(buf.data(), (int64_t)buf.size(), target->shape), target);
}

void Initializer::fill(const Tensor& target, NativeBackend& be, PcgRng& rng) const {
  switch (kind) {
    case InitKind::Zeros: return;
    case InitKind::Ones: be.copy(be.add_scalar(target, 1.0f), target); return;
    case InitKind::Normal: fill_gaussian(target, be, rng, a, b); return;
    case InitKind::Xavier: {
      auto f = fans(target->shape);
      fill_gaussian(target, be, rng, 0.0f, a * sqrtf(2.0f / (float)(f.first + f.second)));
      return;
    }
    case InitKind::Kaiming: {
      auto f = fans(target->shape);
      fill_gaussian(target, be, rng, 0.0f, a / sqrtf((float)f.first));
      return;
    }
  }
}

static Initializer normal(float mean, float std) { return Initializer{InitKind::Normal, mean, std}; }
static Initializer ones() { return Initializer{InitKind::Ones, 0, 0}; }
static Initializer kaiming(float gain = 1.41421356f) { return Initializer{InitKind::Kaiming, gain, 0}; }

void ModelConfig::validate() const {
  if (head_count < 1) throw ArgumentError("HeadCount must be >= 1.");
  if (kv_head_count < 1 || kv_head_count > head_count) throw ArgumentError("KvHeadCount must be in [1, HeadCount].");
  if (head_count % kv_head_count) throw ArgumentError("HeadCount must be divisible by KvHeadCount.");
  if (embedding_dim % head_count) throw ArgumentError("EmbeddingDim must be divisible by HeadCount.");
  if (head_dim() % 2) throw ArgumentError("HeadDim must be even for RoPE.");
}

// ---------------------------------------------------------------- Module (Module.cs:67-123)
Tensor Module::param(const std::string& name, const Dims& shape, Initializer init) {
  Tensor p = be().allocate(shape);
  p->requires_grad = true;
  p->backend = ctx_.backend;
  if (!ctx_.skip_init) {
    GradMode::Guard nograd(true);
    if (ctx_.override_init && shape.size() == 2) init = *ctx_.override_init;
    init.fill(p, be(), *ctx_.rng);
  }
  params_.emplace_back(name, p);
  return p;
}

std::vector<Tensor> Module::parameters() const {
  std::vector<Tensor> out;
  for (const auto& kv : named_parameters()) out.push_back(kv.second);
  return out;
}

std::vector<std::pair<std::string, Tensor>> Module::named_parameters() const {
  std::vector<std::pair<std::string, Tensor>> out(params_.begin(), params_.end());
  for (const auto& c : children_)
    for (const auto& kv : c.second->named_parameters()) out.emplace_back(c.first + "." + kv.first, kv.second);
  return out;
}

// ---------------------------------------------------------------- Linear (Linear.cs:10-43): y = x·Wᵀ
Linear::Linear(ParameterContext ctx, int in, int out, Initializer init) : Module(ctx), in_dim(in), out_dim(out) {
  weight = param("weight", {out, in}, init);
}

Tensor Linear::forward(const Tensor& x) {
  if (x->shape.back() != in_dim) throw ArgumentError("Linear expected last dim " + std::to_string(in_dim) + ", got " + dims_str(x->shape) + ".");
  if (x->rank() == 2) return ag().matmul(x, weight, true);
  int rows = (int)(x->numel() / in_dim);
  Dims lead(x->shape.begin(), x->shape.end() - 1);
  Tensor flat = ag().reshape(ag().contiguous(x), {rows, in_dim});
  Tensor y = ag().matmul(flat, weight, true);
  lead.push_back(out_dim);
  return ag().reshape(y, lead);
}

// ---------------------------------------------------------------- RmsNorm (Modules.cs:6-22)
RmsNorm::RmsNorm(ParameterContext ctx, int dim, float e) : Module(ctx), eps(e) { weight = param("weight", {dim}, ones()); }
Tensor RmsNorm::forward(const Tensor& x) { return ag().rms_norm(x, weight, eps); }

// ---------------------------------------------------------------- RotaryEmbedding (Modules.cs:28-80)
RotaryEmbedding::RotaryEmbedding(ParameterContext ctx, int hd, float theta, int ms) : Module(ctx), max_seq(ms) {
  if (hd % 2) throw ArgumentError("RoPE head dim must be even.");
  int half = hd / 2;
  std::vector<float> c((size_t)ms * hd), s((size_t)ms * hd);
  for (int p = 0; p < ms; p++)
    for (int j = 0; j < half; j++) {
      float freq = 1.0f / powf(theta, (2.0f * (float)j) / (float)hd);
      float angle = (float)p * freq;
      float cv = cosf(angle), sv = sinf(angle);
      c[(size_t)p * hd + j] = cv; c[(size_t)p * hd + j + half] = cv;
      s[(size_t)p * hd + j] = sv; s[(size_t)p * hd + j + half] = sv;
    }
  cos = be().from_host(c.data(), (int64_t)c.size(), {ms, hd});
  sin = be().from_host(s.data(), (int64_t)s.size(), {ms, hd});
  for (auto& v : s) v = -v;
  neg_sin = be().from_host(s.data(), (int64_t)s.size(), {ms, hd});
}

Tensor RotaryEmbedding::apply_at_offset(const Tensor& x, int offset) {
  int seq = x->shape[(size_t)x->rank() - 2];
  if (offset < 0 || offset + seq > max_seq)
    throw OutOfRangeError("RoPE positions " + std::to_string(offset) + ".." + std::to_string(offset + seq - 1) +
                          " exceed the table length " + std::to_string(max_seq) + ".");
  return ag().rotary(x, cos->slice(0, offset, seq), sin->slice(0, offset, seq), neg_sin->slice(0, offset, seq));
}

Tensor RotaryEmbedding::apply_seq_major(const Tensor& x, int offset) {
  if (x->rank() != 4) throw ArgumentError("RoPE on [b, s, heads, dh] expects a rank-4 tensor; got " + dims_str(x->shape) + ".");
  int seq = x->shape[1], hd = x->shape[3];
  if (offset < 0 || offset + seq > max_seq)
    throw OutOfRangeError("RoPE positions " + std::to_string(offset) + ".." + std::to_string(offset + seq - 1) +
                          " exceed the table length " + std::to_string(max_seq) + ".");
  // table rows offset .. offset+seq-1 as [seq, 1, dh]: broadcast over the heads axis
  auto rows = [&](const Tensor& t) { return t->slice(0, offset, seq)->reshape({seq, 1, hd}); };
  return ag().rotary(x, rows(cos), rows(sin), rows(neg_sin));
}

// ---------------------------------------------------------------- SwiGLU (Modules.cs:84-109)
SwiGlu::SwiGlu(ParameterContext ctx, int dim, int hidden) : Module(ctx) {
  gate = register_module("gate", std::make_unique<Linear>(ctx, dim, hidden, kaiming()));
  up = register_module("up", std::make_unique<Linear>(ctx, dim, hidden, kaiming()));
  down = register_module("down", std::make_unique<Linear>(ctx, hidden, dim, kaiming()));
}

Tensor SwiGlu::forward(const Tensor& x) {
  Tensor g = gate->forward(x);
  Tensor u = up->forward(x);
  return down->forward(ag().silu_mul(g, u));
}

// ---------------------------------------------------------------- Attention (Modules.cs:120-219)
Attention::Attention(ParameterContext ctx, const ModelConfig& c, int l) : Module(ctx), cfg(c), layer(l) {
  c.validate();
  int d = c.embedding_dim, h = c.head_count, kvh = c.kv_head_count, dh = c.head_dim();
  wq = register_module("wq", std::make_unique<Linear>(ctx, d, h * dh, normal(0, 0.02f)));
  wk = register_module("wk", std::make_unique<Linear>(ctx, d, kvh * dh, normal(0, 0.02f)));
  wv = register_module("wv", std::make_unique<Linear>(ctx, d, kvh * dh, normal(0, 0.02f)));
  wo = register_module("wo", std::make_unique<Linear>(ctx, h * dh, d, normal(0, 0.02f)));
  rope = register_module("rope", std::make_unique<RotaryEmbedding>(ctx, dh, c.rope_theta, c.max_sequence_length));
  float inv = 1.0f / sqrtf((float)dh);
  inv_sqrt_hd = be().from_host(&inv, 1, {1});
}

Tensor Attention::causal_mask(int q_len, int k_len, int pos_offset) {
  std::vector<float> m((size_t)q_len * k_len);
  for (int i = 0; i < q_len; i++)
    for (int j = 0; j < k_len; j++) m[(size_t)i * k_len + j] = j <= pos_offset + i ? 0.0f : -1e9f;
  return be().from_host(m.data(), (int64_t)m.size(), {q_len, k_len});
}

Tensor Attention::forward(const Tensor& x, const ForwardContext& fctx) {
  KvCache* cache = fctx.cache;
  if (cache && GradMode::enabled()) throw InvalidOperationError("KV-cache decode is inference-only; wrap it in GradMode.NoGrad().");
  int b = x->shape[0], s = x->shape[1];
  int h = cfg.head_count, kvh = cfg.kv_head_count, dh = cfg.head_dim(), g = h / kvh;
  int pos_offset = cache ? cache->length(layer) : 0;
  Autograd& A = ag();
  Tensor qh, kh;
  Tensor vh = A.transpose(A.reshape(wv->forward(x), {b, s, kvh, dh}), 1, 2);
  if (!cache) {
    // RoPE on the projections' [b, s, heads, dh] layout, then the head-major views attention reads. The rotation of
    // each element is the one RotaryEmbedding applies to the head-major view (same pair, same table row), and the
    // backward's rotated gradient comes out dense in [b, s, heads, dh], so folding it back into the projection's
    // [b, s, heads·dh] rows is a reshape, not a copy.
    qh = A.transpose(rope->apply_seq_major(A.reshape(wq->forward(x), {b, s, h, dh}), pos_offset), 1, 2);
    kh = A.transpose(rope->apply_seq_major(A.reshape(wk->forward(x), {b, s, kvh, dh}), pos_offset), 1, 2);
  } else {
    qh = rope->apply_at_offset(A.transpose(A.reshape(wq->forward(x), {b, s, h, dh}), 1, 2), pos_offset);
    kh = rope->apply_at_offset(A.transpose(A.reshape(wk->forward(x), {b, s, kvh, dh}), 1, 2), pos_offset);
  }
  int key_len = s;
  if (cache) {
    auto kv = cache->append(layer, kh, vh);
    kh = kv.first;
    vh = kv.second;
    key_len = pos_offset + s;
  }
  if (be().use_fused && be().has_fused() && dh <= 64) {
    // One fused node: causal online-softmax attention straight into the merged-heads layout [b, s, h, dh].
    Tensor o = A.attention(qh, kh, vh, 1.0f / sqrtf((float)dh), pos_offset);
    return wo->forward(A.reshape(o, {b, s, h * dh}));
  }
  Tensor q5 = A.reshape(A.contiguous(qh), {b, kvh, g, s, dh});
  Tensor k5 = A.reshape(A.contiguous(kh), {b, kvh, 1, key_len, dh});
  Tensor v5 = A.reshape(A.contiguous(vh), {b, kvh, 1, key_len, dh});
  Tensor scores = A.matmul(A.mul(q5, inv_sqrt_hd), k5, true);
  Tensor probs;
  if (s == 1) {
    probs = A.softmax(scores, -1);
  } else {
    probs = A.softmax(A.add(scores, causal_mask(s, key_len, pos_offset)), -1);
  }
  Tensor context = A.matmul(probs, v5);
  Tensor heads = A.reshape(A.contiguous(context), {b, h, s, dh});
  Tensor merged = A.reshape(A.contiguous(A.transpose(heads, 1, 2)), {b, s, h * dh});
  return wo->forward(merged);
}

// ---------------------------------------------------------------- TransformerBlock (Modules.cs:222-246)
TransformerBlock::TransformerBlock(ParameterContext ctx, const ModelConfig& c, int l) : Module(ctx) {
  attn_norm = register_module("attn_norm", std::make_unique<RmsNorm>(ctx, c.embedding_dim, c.norm_eps));
  attn = register_module("attn", std::make_unique<Attention>(ctx, c, l));
  ffn_norm = register_module("ffn_norm", std::make_unique<RmsNorm>(ctx, c.embedding_dim, c.norm_eps));
  ffn = register_module("ffn", std::make_unique<SwiGlu>(ctx, c.embedding_dim, c.ffn_hidden));
}

Tensor TransformerBlock::forward(const Tensor& x, const ForwardContext& fctx) {
  Tensor h = ag().add(x, attn->forward(attn_norm->forward(x), fctx));
  return ag().add(h, ffn->forward(ffn_norm->forward(h)));
}

// ---------------------------------------------------------------- Embedding (Embedding.cs:9-46)
Embedding::Embedding(ParameterContext ctx, int v, int d) : Module(ctx), vocab(v), dim(d) {
  weight = param("weight", {v, d}, normal(0, 0.02f));
}

std::vector<int> ids_from_tensor(NativeBackend& be, const Tensor& t) {
  std::vector<float> host((size_t)t->numel());
  be.to_host(t, host.data(), (int64_t)host.size());
  std::vector<int> ids(host.size());
  for (size_t i = 0; i < host.size(); i++) ids[i] = (int)std::nearbyint(host[i]);  // MathF.Round: ties to even
  return ids;
}

Tensor Embedding::forward(const Tensor& input) {
  std::vector<int> ids = ids_from_tensor(be(), input);
  Tensor rows = ag().embedding(weight, ids);
  if (input->rank() == 1) return rows;
  Dims out = input->shape;
  out.push_back(dim);
  return ag().reshape(rows, out);
}

// ---------------------------------------------------------------- LlamaModel (Modules.cs:252-288)
LlamaModel::LlamaModel(ParameterContext ctx, const ModelConfig& c) : Module(ctx), cfg(c) {
  c.validate();
  embedding = register_module("embedding", std::make_unique<Embedding>(ctx, c.vocab_size, c.embedding_dim));
  for (int i = 0; i < c.layer_count; i++)
    blocks.push_back(register_module("block." + std::to_string(i), std::make_unique<TransformerBlock>(ctx, c, i)));
  final_norm = register_module("final_norm", std::make_unique<RmsNorm>(ctx, c.embedding_dim, c.norm_eps));
}

Tensor LlamaModel::forward(const Tensor& ids, const ForwardContext& fctx) {
  Tensor h = embedding->forward(ids);
  for (size_t i = 0; i < blocks.size(); i++) {
    TransformerBlock* block = blocks[i];
    if (gradient_checkpointing && GradMode::enabled()) {
      std::function<void()> ready;
      if (on_block_grads_ready) {
        int idx = (int)i;
        auto hook = on_block_grads_ready;
        ready = [hook, idx]() { hook(idx); };
      }
      h = ag().checkpoint([block, fctx](const Tensor& x) { return block->forward(x, fctx); }, h, block->parameters(), ready);
    } else {
      h = block->forward(h, fctx);
    }
  }
  h = final_norm->forward(h);
  // tied head MatMul(h, Emb.W, transposeB) (Modules.cs:278-287) on the rows [B·S, D], as Linear flattens its input:
  // the same logits, and the weight gradient comes out of one K = B·S product instead of B per-sequence products
  // summed by ReduceGradToShape
  if (h->rank() == 2) return ag().matmul(h, embedding->weight, true);
  const int d = h->shape.back();
  const int rows = (int)(h->numel() / d);
  Dims lead(h->shape.begin(), h->shape.end() - 1);
  Tensor y = ag().matmul(ag().reshape(ag().contiguous(h), {rows, d}), embedding->weight, true);
  lead.push_back(embedding->weight->shape[0]);
  return ag().reshape(y, lead);
}

// ---------------------------------------------------------------- KvCache (Modules.cs:301-370)
KvCache::KvCache(NativeBackend* be, const ModelConfig& cfg, int mb, int ms)
    : max_batch(mb), max_seq(ms), be_(be), key_store_((size_t)cfg.layer_count), value_store_((size_t)cfg.layer_count),
      lengths_((size_t)cfg.layer_count, 0) {}

int KvCache::length(int layer) const {
  if (layer < 0 || layer >= (int)lengths_.size()) throw OutOfRangeError("layer out of range for the cache");
  return lengths_[(size_t)layer];
}

std::pair<Tensor, Tensor> KvCache::append(int layer, const Tensor& k, const Tensor& v) {
  if (layer < 0 || layer >= (int)key_store_.size()) throw OutOfRangeError("layer out of range for the cache (model/cache config mismatch?)");
  int batch = k->shape[0], new_len = k->shape[2];
  if (batch > max_batch) throw InvalidOperationError("batch exceeds the cache's MaxBatch");
  int len = lengths_[(size_t)layer];
  if (len + new_len > max_seq)
    throw InvalidOperationError("KV cache overflow: " + std::to_string(len + new_len) + " positions exceeds the maximum " +
                                std::to_string(max_seq) + ".");
  Tensor& ks = key_store_[(size_t)layer];
  Tensor& vs = value_store_[(size_t)layer];
  if (!ks) {
    ks = be_->allocate({batch, k->shape[1], max_seq, k->shape[3]});
    vs = be_->allocate({batch, v->shape[1], max_seq, v->shape[3]});
  } else if (ks->shape[0] != batch || ks->shape[1] != k->shape[1] || ks->shape[3] != k->shape[3]) {
    // the reference's Cat along the position axis rejects the same mismatch
    throw ArgumentError("KV cache append: shape [" + std::to_string(batch) + ", " + std::to_string(k->shape[1]) + ", *, " +
                        std::to_string(k->shape[3]) + "] does not match the cached layer");
  }
  be_->copy(k, ks->slice(2, len, new_len));
  be_->copy(v, vs->slice(2, len, new_len));
  lengths_[(size_t)layer] = len + new_len;
  return {ks->slice(2, 0, len + new_len), vs->slice(2, 0, len + new_len)};
}

void KvCache::advance(int positions) {
  for (size_t l = 0; l < lengths_.size(); l++) {
    if (!key_store_[l]) throw InvalidOperationError("KV cache layer " + std::to_string(l) + " has no storage yet (prefill first)");
    if (lengths_[l] + positions > max_seq)
      throw InvalidOperationError("KV cache overflow: " + std::to_string(lengths_[l] + positions) +
                                  " positions exceeds the maximum " + std::to_string(max_seq) + ".");
  }
  for (int& n : lengths_) n += positions;
}

void KvCache::reset() {
  for (auto& t : key_store_) t.reset();
  for (auto& t : value_store_) t.reset();
  std::fill(lengths_.begin(), lengths_.end(), 0);
}

// ---------------------------------------------------------------- Loss (Loss.cs:13-33)
Tensor cross_entropy_loss(Autograd& ag, const Tensor& logits, const Tensor& targets, int ignore) {
  int vocab = logits->shape.back();
  int n = (int)(logits->numel() / vocab);
  Tensor flat = logits->rank() == 2 ? logits : ag.reshape(ag.contiguous(logits), {n, vocab});
  std::vector<int> ids = ids_from_tensor(*ag.be, targets);
  if ((int)ids.size() != n) throw ArgumentError("targets must have one entry per logits row.");
  return ag.cross_entropy(flat, ids, ignore);
}

// ---------------------------------------------------------------- samplers (Sampling.cs:18-112)
int argmax(const float* logits, int n) {
  if (n <= 0) throw ArgumentError("logits must be non-empty.");
  int best = -1;
  float best_val = -INFINITY;
  for (int i = 0; i < n; i++) {
    float v = logits[i];
    if (std::isnan(v)) continue;
    if (best < 0 || v > best_val) { best = i; best_val = v; }
  }
  return best < 0 ? 0 : best;
}

// Sampling.cs:60-84: temperature softmax, then the indices by descending probability (ties by index) cut to top-k and
// top-p. The order is a strict total order, so when top-k bounds the kept set only that prefix is sorted
// (std::partial_sort yields exactly the full sort's first k entries).
void TopKTopPSampler::prepare(const float* logits, int vocab, Prepared& p) const {
  if (vocab <= 0) throw ArgumentError("logits must be non-empty.");
  p.direct = -1;
  if (temperature <= 0.0f) { p.direct = argmax(logits, vocab); return; }
  float mx = -INFINITY;
  for (int i = 0; i < vocab; i++)
    if (logits[i] > mx) mx = logits[i];
  std::vector<float>& probs = p.probs;
  probs.resize((size_t)vocab);
  float sum = 0.0f;
  for (int i = 0; i < vocab; i++) {
    float e = expf((logits[i] - mx) / temperature);
    probs[(size_t)i] = e;
    sum += e;
  }
  if (!std::isfinite(sum) || sum <= 0.0f) { p.direct = argmax(logits, vocab); return; }
  for (int i = 0; i < vocab; i++) probs[(size_t)i] /= sum;
  std::vector<int>& order = p.order;
  order.resize((size_t)vocab);
  std::iota(order.begin(), order.end(), 0);
  auto before = [&](int a, int b) {
    if (probs[(size_t)a] != probs[(size_t)b]) return probs[(size_t)a] > probs[(size_t)b];
    return a < b;
  };
  int keep = vocab;
  if (top_k > 0 && top_k < keep) keep = top_k;
  if (keep < vocab)
    std::partial_sort(order.begin(), order.begin() + keep, order.end(), before);
  else
    std::sort(order.begin(), order.end(), before);
  if (top_p < 1.0f) {
    float cumulative = 0.0f;
    int kept = 0;
    for (int i = 0; i < keep; i++) {
      cumulative += probs[(size_t)order[(size_t)i]];
      kept++;
      if (cumulative >= top_p) break;
    }
    keep = std::max(1, kept);
  }
  p.keep = keep;
}

// Sampling.cs:86-111: one RNG draw over the renormalised kept set.
int TopKTopPSampler::draw(const Prepared& p) {
  if (p.direct >= 0) return p.direct;
  float total = 0.0f;
  for (int i = 0; i < p.keep; i++) total += p.probs[(size_t)p.order[(size_t)i]];
  float r = rng.next_float() * total;
  float acc = 0.0f;
  for (int i = 0; i < p.keep; i++) {
    acc += p.probs[(size_t)p.order[(size_t)i]];
    if (r < acc) return p.order[(size_t)i];
  }
  return p.order[(size_t)p.keep - 1];
}

int TopKTopPSampler::sample(const float* logits, int vocab) {
  Prepared p;
  prepare(logits, vocab, p);
  return draw(p);
}

// Process-wide worker threads for per-row host work, started once (decode samples every step, and starting threads
// per step cost about as much as the work): run(n, fn) calls fn(i) for every i in [0, n) on the workers and the
// calling thread and returns when all are done, rethrowing the first exception. One job runs at a time. The workers
// are detached and never stopped, so process exit does not wait for them.
//
// Fork: a child has only the thread that called fork(), and any mutex another parent thread held at that moment is
// copied locked. A pthread_atfork child handler therefore forgets the parent's pool (its memory is never touched again
// in the child: its locks may be held by threads that do not exist there) and re-creates the creation lock, so the
// child's first instance() starts a pool of its own whichever thread of the parent forked and whatever it held.
namespace {
class RowPool {
 public:
  static RowPool& instance() {
    static std::once_flag hook;
    std::call_once(hook, [] { pthread_atfork(nullptr, nullptr, &RowPool::after_fork_child); });
    std::lock_guard<std::mutex> g(create_lock());
    RowPool*& pool = slot();
    if (!pool) pool = new RowPool((int)std::max(1u, std::thread::hardware_concurrency()) - 1);
    return *pool;
  }

  void run(int n, const std::function<void(int)>& fn) {
    std::lock_guard<std::mutex> job(job_mu_);
    {
      std::lock_guard<std::mutex> g(mu_);
      fn_ = &fn;
      n_ = n;
      next_.store(0);
      done_ = 0;
      err_ = nullptr;
      gen_++;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> g(mu_);
    done_cv_.wait(g, [&] { return done_ == workers_; });  // every worker has finished this job
    fn_ = nullptr;
    if (err_) std::rethrow_exception(err_);
  }

 private:
  static std::mutex& create_lock() {
    static std::mutex m;
    return m;
  }
  static RowPool*& slot() {
    static RowPool* p = nullptr;
    return p;
  }
  static void after_fork_child() {
    new (&create_lock()) std::mutex();  // unlocked again, whatever its state at the fork
    slot() = nullptr;                   // the parent's pool stays allocated and unused
  }

  explicit RowPool(int workers) : workers_(workers) {
    for (int i = 0; i < workers; i++) std::thread([this] { loop(); }).detach();
  }

  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] { return gen_ != seen; });
        seen = gen_;
      }
      work();
      {
        std::lock_guard<std::mutex> g(mu_);
        done_++;
      }
      done_cv_.notify_one();
    }
  }

  void work() {
    for (int i = next_.fetch_add(1); i < n_; i = next_.fetch_add(1)) {
      try {
        (*fn_)(i);
      } catch (...) {
        std::lock_guard<std::mutex> g(mu_);
        if (!err_) err_ = std::current_exception();
      }
    }
  }

  const int workers_;
  std::mutex job_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int)>* fn_ = nullptr;
  int n_ = 0;
  std::atomic<int> next_{0};
  int done_ = 0;
  uint64_t gen_ = 0;
  std::exception_ptr err_;
};
}  // namespace

void TopKTopPSampler::sample_rows(const float* rows, int batch, int vocab, int* out) {
  if (rows_.size() < (size_t)batch) rows_.resize((size_t)batch);
  std::vector<Prepared>& prep = rows_;
  if (batch <= 1) {
    for (int b = 0; b < batch; b++) prepare(rows + (size_t)b * vocab, vocab, prep[(size_t)b]);
  } else {
    // rows are independent: prepared in any order on the pool; the draws below stay in row order
    RowPool::instance().run(batch, [&](int b) { prepare(rows + (size_t)b * vocab, vocab, prep[(size_t)b]); });
  }
  for (int b = 0; b < batch; b++) out[b] = draw(prep[(size_t)b]);
}

}  // namespace paihost
