// AdamW (ProjectAI.Core/Optimizers.cs:14-133), the training step of Trainer.Train (ProjectAI.Training/Training.cs:59-120)
// with its warmup+cosine schedule (:165-181), data-parallel gradient buckets, and the decode loop of
// Inference.GenerateText (Inference.cs:23-74).
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <filesystem>
#include <memory>

#include "runtime.h"

namespace paihost {

AdamW::AdamW(std::vector<Tensor> params, NativeBackend* be, float lr_, float b1_, float b2_, float eps_, float wd_)
    : lr(lr_), b1(b1_), b2(b2_), eps(eps_), wd(wd_), params_(std::move(params)), be_(be) {}

// This rank's shard of a flattened parameter (or gradient): elements [r·n/W, (r+1)·n/W).
static Tensor shard_of(const Tensor& t, int rank, int world) {
  const int64_t n = t->numel(), s = n / world;
  return t->reshape({(int)n})->slice(0, (int)(rank * s), (int)s);
}

// AdamW.Step (Optimizers.cs:81-123). The fused path runs the same per-element operations in one kernel, in place.
// Under ZeRO-1 (shard_world > 1) a shardable parameter is updated through views of its shard (the same element
// operations on fewer elements), with moments of the shard's size.
void AdamW::step() {
  step_count++;
  float cur_lr = schedule ? schedule(step_count) : lr;
  GradMode::Guard nograd(true);
  bool fused = be_->use_fused && be_->has_fused();
  if (fused) {
    for (const auto& p : params_) {
      if (!p->grad) continue;
      State& s = state[p.get()];
      const bool sh = sharded(p);
      const Tensor pv = sh ? shard_of(p, shard_rank, shard_world) : p;
      const Tensor gv = sh ? shard_of(p->grad, shard_rank, shard_world) : p->grad;
      if (!s.m) {
        s.m = be_->allocate(pv->shape);  // zero-initialised moments, persisting across steps
        s.v = be_->allocate(pv->shape);
        be_->keep_alive(s.m);
        be_->keep_alive(s.v);
      }
      s.t += 1;
      be_->adamw_step(pv, gv, s.m, s.v, cur_lr, b1, b2, eps, wd, s.t, grad_scale);
    }
    return;
  }
  be_->begin_scope();
  try {
    for (const auto& param : params_) {
      if (!param->grad) continue;
      const bool sh = sharded(param);
      const Tensor p = sh ? shard_of(param, shard_rank, shard_world) : param;
      Tensor g = sh ? shard_of(param->grad, shard_rank, shard_world) : param->grad;
      if (grad_scale != 1.0f) g = be_->mul_scalar(g, grad_scale);
      State& s = state[param.get()];
      Tensor prev_m = s.m, prev_v = s.v;
      if (!s.m) s.m = be_->allocate(p->shape);
      if (!s.v) s.v = be_->allocate(p->shape);
      int t = s.t + 1;
      Tensor m = be_->add(be_->mul_scalar(s.m, b1), be_->mul_scalar(g, 1.0f - b1));
      Tensor v = be_->add(be_->mul_scalar(s.v, b2), be_->mul_scalar(be_->mul(g, g), 1.0f - b2));
      s.m = m;
      s.v = v;
      s.t = t;
      be_->keep_alive(m);
      be_->keep_alive(v);
      if (prev_m) be_->release(prev_m);
      if (prev_v) be_->release(prev_v);
      float bc1 = 1.0f - powf(b1, (float)t);
      float bc2 = 1.0f - powf(b2, (float)t);
      Tensor mhat = be_->mul_scalar(m, 1.0f / bc1);
      Tensor vhat = be_->mul_scalar(v, 1.0f / bc2);
      Tensor adaptive = be_->div(mhat, be_->add_scalar(be_->sqrt(vhat), eps));
      Tensor delta = be_->add(be_->mul_scalar(adaptive, cur_lr), be_->mul_scalar(p, cur_lr * wd));
      be_->copy(be_->sub(p, delta), p);
    }
  } catch (...) {
    be_->end_scope();
    throw;
  }
  be_->end_scope();
}

void AdamW::zero_grad() {
  for (const auto& p : params_) {
    if (p->grad) be_->release(p->grad);
    p->grad.reset();
  }
}

std::function<float(int)> warmup_cosine(const TrainingConfig& cfg) {
  float base = cfg.learning_rate, min_lr = base * 0.1f;
  int total = std::max(1, cfg.max_steps);
  int warmup = std::min(std::max(cfg.warmup_steps, 0), std::max(0, total - 1));
  return [=](int step) {
    if (warmup > 0 && step <= warmup) return base * (float)step / (float)warmup;
    float denom = (float)std::max(1, total - warmup);
    float progress = std::min(std::max((float)(step - warmup) / denom, 0.0f), 1.0f);
    float cosine = 0.5f * (1.0f + cosf(3.14159265f * progress));
    return min_lr + (base - min_lr) * cosine;
  };
}

Trainer::Trainer(NativeBackend* be, LlamaModel* m, const TrainingConfig& c, float beta1, float beta2)
    : model(m), cfg(c), ag(be), be_(be) {
  model->gradient_checkpointing = cfg.gradient_checkpointing;
  params_ = model->parameters();
  optimizer = std::make_unique<AdamW>(params_, be, cfg.learning_rate, beta1, beta2, 1e-8f, cfg.weight_decay);
  optimizer->schedule = warmup_cosine(cfg);
  for (auto* b : model->blocks) block_params_.push_back(b->parameters());
  tail_params_ = model->embedding->parameters();
  for (const auto& p : model->final_norm->parameters()) tail_params_.push_back(p);
}

static std::vector<Tensor> grads_of(const std::vector<Tensor>& params) {
  std::vector<Tensor> g;
  for (const auto& p : params)
    if (p->grad) g.push_back(p->grad);
  return g;
}

// Host buffers in (NextBatch's FromHost, Training.cs:122-141), host loss out: the end-to-end step.
float Trainer::step(const std::vector<std::vector<float>>& inputs, const std::vector<std::vector<float>>& targets) {
  int b = cfg.batch_size, s = cfg.sequence_length;
  if (inputs.size() != targets.size() || inputs.empty())
    throw ArgumentError("inputs and targets must hold the same number (>= 1) of micro-batches");
  std::vector<Tensor> in, tg;
  for (size_t i = 0; i < inputs.size(); i++) {
    if ((int64_t)inputs[i].size() != (int64_t)b * s || (int64_t)targets[i].size() != (int64_t)b * s)
      throw ArgumentError("each micro-batch must hold batch_size x sequence_length ids");
    in.push_back(be_->from_host(inputs[i].data(), (int64_t)b * s, {b, s}));
    tg.push_back(be_->from_host(targets[i].data(), (int64_t)b * s, {b, s}));
  }
  return step_tensors(in, tg);
}

int Trainer::configure_shards() {
  const int ranks = world > 0 ? world : be_->dp_world;
  const int my_rank = rank >= 0 ? rank : be_->dp_rank;
  const bool shard = ranks > 1 && zero1;
  optimizer->shard_world = shard ? ranks : 1;
  optimizer->shard_rank = shard ? my_rank : 0;
  return ranks;
}

float Trainer::step_tensors(const std::vector<Tensor>& inputs, const std::vector<Tensor>& targets) {
  int micro_steps = std::max(1, (int)inputs.size());
  if ((int)targets.size() != micro_steps) throw ArgumentError("inputs and targets must hold the same number of micro-batches");
  const int ranks = configure_shards();
  const bool dp = ranks > 1;
  const bool shard = dp && zero1;
  auto exchange = [this, shard](const std::vector<Tensor>& g) {
    if (g.empty()) return;
    std::vector<Tensor> whole, split;
    for (const auto& t : g) (shard && t->numel() % optimizer->shard_world == 0 ? split : whole).push_back(t);
    if (!whole.empty()) {
      if (allreduce) allreduce(whole);
      else be_->allreduce(whole);
    }
    if (!split.empty()) {
      if (reduce_scatter) reduce_scatter(split);
      else be_->reduce_scatter(split);
    }
  };
  optimizer->grad_scale = dp ? 1.0f / (float)ranks : 1.0f;
  optimizer->zero_grad();
  float inv_micro_v = 1.0f / (float)micro_steps;
  Tensor inv_micro = be_->from_host(&inv_micro_v, 1, {1});
  float step_loss = 0.0f;
  for (int micro = 0; micro < micro_steps; micro++) {
    bool last = micro == micro_steps - 1;
    // Data parallel: each checkpointed block's gradients are final once its recompute ran; sum them across ranks
    // right away so the exchange overlaps the backward of the earlier blocks.
    if (dp && last && model->gradient_checkpointing) {
      model->on_block_grads_ready = [this, exchange](int i) { exchange(grads_of(block_params_[(size_t)i])); };
    } else {
      model->on_block_grads_ready = nullptr;
    }
    be_->begin_scope();
    try {
      const Tensor& input = inputs[(size_t)micro];
      const Tensor& target = targets[(size_t)micro];
      Tensor logits = model->forward(input);
      Tensor loss = cross_entropy_loss(ag, logits, target);
      float lh = 0.0f;
      be_->to_host(loss, &lh, 1);
      step_loss += lh / (float)micro_steps;
      Tensor scaled = micro_steps > 1 ? ag.mul(loss, inv_micro) : loss;
      scaled->backward();
      for (const auto& p : params_)
        if (p->grad) be_->keep_alive(p->grad);
    } catch (...) {
      model->on_block_grads_ready = nullptr;
      be_->end_scope();
      throw;
    }
    be_->end_scope();
  }
  model->on_block_grads_ready = nullptr;
  if (dp) {
    if (model->gradient_checkpointing) {
      exchange(grads_of(tail_params_));
    } else {
      exchange(grads_of(params_));
    }
    if (allreduce_wait) allreduce_wait();
    else if (!allreduce) be_->allreduce_wait();
  }
  optimizer->step();
  if (shard) {
    // every rank updated its shards: gather them so all replicas hold the full new parameters
    std::vector<Tensor> split;
    for (const auto& p : params_)
      if (p->grad && optimizer->sharded(p)) split.push_back(p);
    if (allgather) allgather(split);
    else be_->allgather(split);
    if (allreduce_wait) allreduce_wait();
    else if (!allgather) be_->allreduce_wait();
  }
  return step_loss;
}

// ---------------------------------------------------------------- GraphDecoder
GraphDecoder::GraphDecoder(NativeBackend* be, LlamaModel* model, KvCache* cache, int batch)
    : be_(be), model_(model), cache_(cache), batch_(batch) {
  if (!be->has_graphs()) throw InvalidOperationError("the backend has no graph decode entry points");
  ids_ = be->allocate({batch});
  pos_ = be->allocate({1});
}

GraphDecoder::~GraphDecoder() {
  if (graph_) {
    try {
      be_->graph_destroy(graph_);
    } catch (...) {
    }
  }
}

// The decode step of LlamaModel::forward for [batch, 1] ids with the cache (TransformerBlock::forward, Attention::forward
// with the fused attention, SwiGlu::forward), each op on the same backend kernels; only the position-dependent ops read
// the position from pos_.
Tensor GraphDecoder::body() {
  NativeBackend& be = *be_;
  const ModelConfig& c = model_->cfg;
  const int b = batch_, h = c.head_count, kvh = c.kv_head_count, dh = c.head_dim(), d = c.embedding_dim;
  const float scale = 1.0f / sqrtf((float)dh);
  Tensor x = be.gather_dev(model_->embedding->weight, ids_);  // [b, d]
  for (size_t l = 0; l < model_->blocks.size(); l++) {
    TransformerBlock* blk = model_->blocks[l];
    Attention* at = blk->attn;
    Tensor hn = be.rms_norm(x, blk->attn_norm->weight, blk->attn_norm->eps);
    Tensor q = be.matmul(hn, at->wq->weight, true)->reshape({b, 1, h, dh})->transpose(1, 2);
    Tensor k = be.matmul(hn, at->wk->weight, true)->reshape({b, 1, kvh, dh})->transpose(1, 2);
    Tensor v = be.matmul(hn, at->wv->weight, true)->reshape({b, 1, kvh, dh})->transpose(1, 2);
    q = be.rotary_at(q, at->rope->cos, at->rope->sin, pos_);
    k = be.rotary_at(k, at->rope->cos, at->rope->sin, pos_);
    Tensor kc = cache_->key_store((int)l), vc = cache_->value_store((int)l);
    be.kv_append(k, v, kc, vc, pos_);
    Tensor o = be.sdpa_decode(q, kc, vc, pos_, scale);  // [b, 1, h, dh]
    x = be.add(x, be.matmul(o->reshape({b, h * dh}), at->wo->weight, true));
    Tensor hf = be.rms_norm(x, blk->ffn_norm->weight, blk->ffn_norm->eps);
    SwiGlu* f = blk->ffn;
    Tensor a = be.silu_mul(be.matmul(hf, f->gate->weight, true), be.matmul(hf, f->up->weight, true));
    x = be.add(x, be.matmul(a, f->down->weight, true));
  }
  x = be.rms_norm(x, model_->final_norm->weight, model_->final_norm->eps);
  return be.matmul(x, model_->embedding->weight, true)->reshape({b, 1, c.vocab_size});
}

// The same step with the fused decode ops, 5 launches per block: RMSNorm + q/k/v products in one pass, RoPE + cache
// append + attention, o-projection + residual, RMSNorm + gate/up products with SiLU·mul, down-projection + residual.
Tensor GraphDecoder::body_fused() {
  NativeBackend& be = *be_;
  const ModelConfig& c = model_->cfg;
  const int b = batch_, h = c.head_count, kvh = c.kv_head_count, dh = c.head_dim();
  const float scale = 1.0f / sqrtf((float)dh);
  const int64_t width = (int64_t)(h + 2 * kvh) * dh;  // columns of the fused q|k|v product
  Tensor x = be.gather_dev(model_->embedding->weight, ids_);  // [b, d]
  for (size_t l = 0; l < model_->blocks.size(); l++) {
    TransformerBlock* blk = model_->blocks[l];
    Attention* at = blk->attn;
    Tensor qkv = be.linear_fused(x, {at->wq->weight, at->wk->weight, at->wv->weight}, 0, nullptr, blk->attn_norm->weight,
                                 blk->attn_norm->eps);  // RmsNorm(x) · [wq; wk; wv]ᵀ: [b, width]
    // views of one position per sequence: [b, heads, 1, dh] inside each row of qkv
    Tensor q = make_view(*qkv, {b, h, 1, dh}, {width, dh, width, 1}, 0);
    Tensor k = make_view(*qkv, {b, kvh, 1, dh}, {width, dh, width, 1}, (int64_t)h * dh);
    Tensor v = make_view(*qkv, {b, kvh, 1, dh}, {width, dh, width, 1}, (int64_t)(h + kvh) * dh);
    Tensor kc = cache_->key_store((int)l), vc = cache_->value_store((int)l);
    Tensor o = be.attn_decode_step(q, k, v, at->rope->cos, at->rope->sin, kc, vc, pos_, scale);  // [b, 1, h, dh]
    x = be.linear_fused(o->reshape({b, h * dh}), {at->wo->weight}, 1, x);
    SwiGlu* f = blk->ffn;
    Tensor a = be.linear_fused(x, {f->gate->weight, f->up->weight}, 2, nullptr, blk->ffn_norm->weight, blk->ffn_norm->eps);
    x = be.linear_fused(a, {f->down->weight}, 1, x);
  }
  Tensor logits = be.linear_fused(x, {model_->embedding->weight}, 0, nullptr, model_->final_norm->weight,
                                  model_->final_norm->eps);
  return logits->reshape({b, 1, c.vocab_size});
}

Tensor GraphDecoder::step(const std::vector<int>& ids) {
  const ModelConfig& c = model_->cfg;
  if ((int)ids.size() != batch_) throw ArgumentError("GraphDecoder: one id per sequence expected");
  for (int id : ids)
    if (id < 0 || id >= c.vocab_size)
      throw OutOfRangeError("id out of range [0," + std::to_string(c.vocab_size) + "). (Parameter 'ids') Actual value was " +
                            std::to_string(id) + ".");
  int pos = cache_->length(0);
  if (pos + 1 > cache_->max_seq)
    throw InvalidOperationError("KV cache overflow: " + std::to_string(pos + 1) + " positions exceeds the maximum " +
                                std::to_string(cache_->max_seq) + ".");
  if (!cache_->key_store(0) || cache_->key_store(0)->shape[0] != batch_)
    throw InvalidOperationError("GraphDecoder: the cache must hold a prefill of the same batch");
  std::vector<float> fid(ids.begin(), ids.end());
  float fpos = (float)pos;
  be_->write(ids_, fid.data(), batch_);
  be_->write(pos_, &fpos, 1);
  const bool use_fused = fused && be_->has_decode_fusions();
  auto run = [&]() { return use_fused ? body_fused() : body(); };
  if (steps_ == 0) {
    logits_ = run();  // eager: every block size the step needs is now in the allocator's cache
  } else if (!graph_) {
    logits_.reset();
    be_->graph_begin();
    try {
      logits_ = run();
    } catch (...) {
      try {
        be_->graph_destroy(be_->graph_end());
      } catch (...) {
      }
      throw;
    }
    graph_ = be_->graph_end();
    be_->graph_launch(graph_);
  } else {
    be_->graph_launch(graph_);
  }
  cache_->advance(1);
  steps_++;
  return logits_;
}

static bool decode_graphs_enabled() {
  const char* e = getenv("PAI_DECODE_GRAPH");
  return !(e && e[0] == '0');
}

// Inference.GenerateText (Inference.cs:23-64) on token ids, for a lockstep batch (KvCache supports uniform batches).
// Only each row's last logits row is read back (SampleLast reads exactly that row of the full download).
GenerateResult generate(NativeBackend* be, LlamaModel* model, const std::vector<int>& prompt, int max_tokens,
                        TopKTopPSampler* sampler, int batch) {
  using clock = std::chrono::steady_clock;
  GenerateResult r;
  const ModelConfig& cfg = model->cfg;
  int p_len = (int)prompt.size() / batch;
  if (p_len * batch != (int)prompt.size() || p_len == 0) throw ArgumentError("prompt must hold batch x length ids");
  KvCache cache(be, cfg, batch, cfg.max_sequence_length);
  ForwardContext ctx;
  ctx.cache = &cache;
  GradMode::Guard nograd(true);
  int vocab = cfg.vocab_size;
  std::vector<float> last_rows((size_t)batch * vocab);
  const bool device_argmax = !sampler && be->has_argmax_rows();
  std::vector<float> picked((size_t)batch);
  auto pick = [&](const Tensor& logits, std::vector<int>& out) {
    int rows = logits->shape[1];
    out.clear();
    out.resize((size_t)batch);
    if (device_argmax) {
      // greedy: the argmax of every sequence's last row on the device (ArgMax's rules), one index per sequence back
      be->to_host(be->argmax_rows(logits->slice(1, rows - 1, 1)), picked.data(), (int64_t)batch);
      for (int bi = 0; bi < batch; bi++) out[(size_t)bi] = (int)picked[(size_t)bi];
      return;
    }
    // one download of every sequence's last row [batch, vocab]; rows are then sampled in batch order
    be->to_host(logits->slice(1, rows - 1, 1), last_rows.data(), (int64_t)last_rows.size());
    if (sampler) {
      sampler->sample_rows(last_rows.data(), batch, vocab, out.data());
    } else {
      for (int bi = 0; bi < batch; bi++) out[(size_t)bi] = argmax(last_rows.data() + (size_t)bi * vocab, vocab);
    }
  };
  auto t0 = clock::now();
  std::vector<float> pf(prompt.begin(), prompt.end());
  Tensor logits = model->forward(be->from_host(pf.data(), (int64_t)pf.size(), {batch, p_len}), ctx);
  std::vector<int> next;
  pick(logits, next);
  auto t1 = clock::now();
  r.prefill_seconds = std::chrono::duration<double>(t1 - t0).count();
  // the per-token steps replay one captured CUDA graph when the backend supports it (dense head dim <= 64 and at most
  // 16 query rows per kv head, the decode attention kernel's range)
  std::unique_ptr<GraphDecoder> graph;
  if (be->has_graphs() && decode_graphs_enabled() && cfg.head_dim() <= 64 && cfg.head_dim() % 4 == 0 &&
      cfg.head_count / cfg.kv_head_count <= 16)
    graph = std::make_unique<GraphDecoder>(be, model, &cache, batch);
  for (int produced = 0; produced < max_tokens; produced++) {
    for (int v : next) r.tokens.push_back(v);
    if (produced + 1 >= max_tokens || p_len + produced + 1 >= cfg.max_sequence_length) break;
    if (graph) {
      logits = graph->step(next);
    } else {
      std::vector<float> step(next.begin(), next.end());
      logits = model->forward(be->from_host(step.data(), batch, {batch, 1}), ctx);
    }
    pick(logits, next);
  }
  r.graph = graph && graph->captured();
  be->sync();
  r.decode_seconds = std::chrono::duration<double>(clock::now() - t1).count();
  return r;
}

}  // namespace paihost

namespace paihost {

// Checkpointing.EnumerateState (Checkpointing.cs:103-115): each parameter by name, then its AdamW moments. Moments
// that ZeRO-1 keeps as one shard per rank are all-gathered into full-size tensors first, so the state has the layout
// and values of a replicated run's.
std::vector<std::pair<std::string, Tensor>> Trainer::state_items() {
  configure_shards();
  const int W = optimizer->shard_world, r = optimizer->shard_rank;
  std::vector<std::pair<std::string, Tensor>> items;
  std::vector<Tensor> gather;
  for (const auto& kv : model->named_parameters()) {
    items.push_back(kv);
    auto it = optimizer->state.find(kv.second.get());
    if (it == optimizer->state.end() || !it->second.m || !it->second.v) continue;
    Tensor m = it->second.m, v = it->second.v;
    if (optimizer->sharded(kv.second) && m->numel() * W == kv.second->numel()) {
      Tensor fm = be_->allocate(kv.second->shape), fv = be_->allocate(kv.second->shape);
      be_->copy(m, shard_of(fm, r, W));
      be_->copy(v, shard_of(fv, r, W));
      gather.push_back(fm);
      gather.push_back(fv);
      m = fm;
      v = fv;
    }
    items.emplace_back("opt.m::" + kv.first, m);
    items.emplace_back("opt.v::" + kv.first, v);
  }
  if (!gather.empty()) {
    // every rank holds the same sharded parameters in the same order, so the gathers pair up across ranks
    if (allgather) allgather(gather);
    else be_->allgather(gather);
    if (allreduce_wait) allreduce_wait();
    else if (!allgather) be_->allreduce_wait();
  }
  return items;
}

void Trainer::save_checkpoint(const std::string& path, int step, const std::string& metadata) {
  be_->begin_scope();  // the gathered moments are released once the library has snapshotted them
  try {
    auto items = state_items();
    if (!(path.empty() && optimizer->shard_world > 1)) be_->save_checkpoint(path, step, items, metadata);
  } catch (...) {
    be_->end_scope();
    throw;
  }
  be_->end_scope();
}

void Trainer::wait_checkpoint() { be_->wait_checkpoint(); }

// Checkpointing.ApplyWeights then ApplyOptimizer (Checkpointing.cs:118-142). Under ZeRO-1 a sharded parameter's
// saved (full-size) moments must hold as many elements as the parameter; this rank keeps its shard of them.
void apply_weights(NativeBackend* be, LlamaModel* model, const std::vector<std::pair<std::string, Tensor>>& items) {
  std::map<std::string, Tensor> dict(items.begin(), items.end());
  for (const auto& kv : model->named_parameters()) {
    auto it = dict.find(kv.first);
    if (it == dict.end()) throw InvalidDataError("checkpoint is missing parameter '" + kv.first + "'.");
    if (it->second->shape != kv.second->shape)
      throw InvalidDataError("checkpoint parameter '" + kv.first + "' shape " + dims_str(it->second->shape) +
                             " != model " + dims_str(kv.second->shape) + ".");
    be->copy(it->second, kv.second);
  }
}

void Trainer::apply_state(const std::vector<std::pair<std::string, Tensor>>& items, int step) {
  configure_shards();
  const int W = optimizer->shard_world, r = optimizer->shard_rank;
  std::map<std::string, Tensor> dict(items.begin(), items.end());
  const auto named = model->named_parameters();
  apply_weights(be_, model, items);
  for (const auto& kv : named) {
    auto m = dict.find("opt.m::" + kv.first), v = dict.find("opt.v::" + kv.first);
    if (m == dict.end() || v == dict.end()) continue;
    Tensor ms = m->second, vs = v->second;
    if (optimizer->sharded(kv.second)) {
      if (ms->numel() != kv.second->numel() || vs->numel() != kv.second->numel())
        throw InvalidDataError("checkpoint moments of '" + kv.first + "' hold " + std::to_string(ms->numel()) + " / " +
                               std::to_string(vs->numel()) + " elements, the parameter " +
                               std::to_string(kv.second->numel()) + "; a sharded optimizer needs full-size moments.");
      ms = shard_of(ms, r, W);
      vs = shard_of(vs, r, W);
    }
    AdamW::State& s = optimizer->state[kv.second.get()];
    if (!s.m || s.m->shape != ms->shape) {
      s.m = be_->allocate(ms->shape);
      be_->keep_alive(s.m);
    }
    if (!s.v || s.v->shape != vs->shape) {
      s.v = be_->allocate(vs->shape);
      be_->keep_alive(s.v);
    }
    be_->copy(ms, s.m);
    be_->copy(vs, s.v);
    s.t = step;  // every parameter is updated every step (dense LM training), as the reference assumes
  }
  optimizer->step_count = step;
}

// NextBatch (Training.cs:122-141) over host sequences: each drawn row's first seq + 1 ids.
std::pair<Tensor, Tensor> HostSequences::batch(NativeBackend* be, const std::vector<int64_t>& rows, int seq) {
  const int b = (int)rows.size();
  std::vector<float> in((size_t)b * seq), tg((size_t)b * seq);
  for (int r = 0; r < b; r++) {
    const auto& s = seqs.at((size_t)rows[(size_t)r]);
    if ((int64_t)s.size() < (int64_t)seq + 1)
      throw InvalidOperationError("dataset sequence " + std::to_string(rows[(size_t)r]) + " has length " +
                                  std::to_string(s.size()) + "; need " + std::to_string(seq + 1) +
                                  " for sequence length " + std::to_string(seq) + ".");
    for (int t = 0; t < seq; t++) {
      in[(size_t)r * seq + t] = (float)s[(size_t)t];
      tg[(size_t)r * seq + t] = (float)s[(size_t)t + 1];
    }
  }
  return {be->from_host(in.data(), (int64_t)in.size(), {b, seq}), be->from_host(tg.data(), (int64_t)tg.size(), {b, seq})};
}

std::pair<Tensor, Tensor> PackedSequences::batch(NativeBackend* be, const std::vector<int64_t>& rows, int seq) {
  auto b = be->dataset_batch(rows);
  if (b.first->rank() != 2 || b.first->shape[1] != seq)
    throw InvalidOperationError("the open dataset holds sequences of length " +
                                std::to_string(b.first->rank() == 2 ? b.first->shape[1] : -1) +
                                "; the training sequence length is " + std::to_string(seq) + ".");
  return b;
}

TrainingReport Trainer::train(SequenceSource& data, const std::function<void(int, float)>& on_step) {
  if (data.count() == 0) throw ArgumentError("dataset is empty. (Parameter 'dataset')");
  const int ranks = configure_shards();
  const int my_rank = rank >= 0 ? rank : be_->dp_rank;
  const bool writer = my_rank == 0, gather = ranks > 1 && zero1;
  const std::string& dir = cfg.checkpoint_directory;
  if (!dir.empty() && writer) {
    std::error_code ec;
    std::filesystem::create_directories(dir, ec);
    if (ec) throw FileIOError("could not create the checkpoint directory '" + dir + "': " + ec.message());
  }
  auto save = [&](int step) {
    if (dir.empty()) return;
    const std::string path = (std::filesystem::path(dir) / ("step-" + std::to_string(step) + ".ckpt")).string();
    if (gather) save_checkpoint(writer ? path : std::string(), step);  // collective: every rank gathers its shards
    else if (writer) save_checkpoint(path, step);
  };
  PcgRng rng = my_rank > 0 ? PcgRng(cfg.seed, 0xDA3E39CB94B95BDBull + (uint64_t)my_rank) : PcgRng(cfg.seed);
  const int micro = std::max(1, cfg.grad_accum);
  const uint32_t n = (uint32_t)data.count();
  TrainingReport report;
  report.step_losses.reserve((size_t)std::max(0, cfg.max_steps));
  for (int step = 1; step <= cfg.max_steps; step++) {
    // The reference draws each micro-batch after the previous one's backward; the draws depend on the generator
    // alone, so drawing the step's micro-batches first gives the same rows in the same order.
    std::vector<Tensor> in, tg;
    for (int m = 0; m < micro; m++) {
      std::vector<int64_t> rows((size_t)cfg.batch_size);
      for (auto& r : rows) r = (int64_t)(rng.next_u32() % n);
      auto b = data.batch(be_, rows, cfg.sequence_length);
      in.push_back(b.first);
      tg.push_back(b.second);
    }
    const float loss = step_tensors(in, tg);
    report.step_losses.push_back(loss);
    if (on_step) on_step(step, loss);
    if (cfg.checkpoint_every_steps > 0 && step % cfg.checkpoint_every_steps == 0) save(step);
  }
  save(cfg.max_steps);  // the final checkpoint
  if (!dir.empty()) wait_checkpoint();
  report.final_step = cfg.max_steps;
  return report;
}

// Trainer.Restore (Training.cs:156-162).
int Trainer::restore(const std::string& path) {
  be_->wait_checkpoint();  // a save of this process still writing the file finishes first
  be_->begin_scope();
  try {
    auto ck = be_->load_checkpoint(path);
    apply_state(ck.tensors, ck.step);
    be_->end_scope();
    return ck.step;
  } catch (...) {
    be_->end_scope();
    throw;
  }
}

}  // namespace paihost
