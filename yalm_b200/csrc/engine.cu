// Decode engine: one GPU (or one tensor-parallel rank), a fixed .yalm architecture, one stream.
//
// Per step the engine replays one CUDA graph (separate graphs for the two InferenceModes, like
// yalm's hydrate/output graphs, src/model.h:134-136).  The graph is
//   step kernel (token/pos in its node parameters; writes positions + embedding row)
//   per layer: QKV matvec (+RMSNorm, clip, RoPE, KV append, sink rotation)
//              -> attention -> wo matvec (+residual) -> gate/up matvec (+RMSNorm, SwiGLU)
//              -> w2 matvec (+residual)
//   [logits mode] classifier matvec (+final RMSNorm)
// with programmatic-dependent-launch edges between consecutive kernels.  Under tensor parallelism
// the wo/w2 matvecs push their partial rows into every rank's exchange slots over NVLink peer
// memory and the following matvec adds them up (no separate collective kernel).
#include "engine.h"
#include "loader.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace yb {

static thread_local std::string t_last_error;
int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
const std::string& last_error() { return t_last_error; }

__global__ void step_kernel(const StepArgs a) {
  pdl_trigger();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    // src/infer.cpp:489-494
    StepState s;
    s.token = a.token;
    s.pos = a.pos;
    s.kv_sink = a.pos >= a.max_seq_len ? 2 : 0;
    s.kv_pos = s.kv_sink + (a.pos - s.kv_sink) % (a.max_seq_len - s.kv_sink);
    s.kv_len = a.pos >= a.max_seq_len ? a.max_seq_len : a.pos + 1;
    s.epoch = a.epoch;
    s.lepoch = a.lepoch;
    s.pad = 0;
    s.sample_op = a.sample_op;
    s.sample_target = a.sample_target;
    s.temperature = a.temperature;
    s.coin = a.coin;
    *a.step = s;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n_bar; i += gridDim.x * blockDim.x) a.bar[i] = 0u;
  // embedding row -> fp32 residual stream (src/infer.cpp:460-481); an fp8 E5M2 value is the top
  // byte of the fp16 with the same value
  if (a.esz == 1) {
    const unsigned char* row = reinterpret_cast<const unsigned char*>(a.emb) + (size_t)a.token * a.dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.dim; i += gridDim.x * blockDim.x)
      a.x[i] = __half2float(__ushort_as_half((unsigned short)(row[i] << 8)));
  } else {
    const __half* row = a.emb + (size_t)a.token * a.dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.dim; i += gridDim.x * blockDim.x)
      a.x[i] = __half2float(row[i]);
  }
}

// Kernel that waits (bounded) for every rank's slice of the gathered logits.
__global__ void tp_gather_wait_kernel(const StepState* step, const unsigned* counters, int tp_size, int grid,
                                      unsigned* status) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x < tp_size) wait_counter_geq(counters + threadIdx.x, step->lepoch * (unsigned)grid, status);
}

namespace {

template <typename T>
int dev_alloc(yb_engine* e, T** p, size_t bytes) {
  void* v = nullptr;
  cudaError_t err = cudaMalloc(&v, bytes ? bytes : 16);
  if (err != cudaSuccess) return set_error(YB_E_CUDA, std::string("cudaMalloc(") + std::to_string(bytes) + ") failed: " + cudaGetErrorString(err));
  e->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return 0;
}

int check_config(const yb_config* c, int tp_size) {
  if (!c) return set_error(YB_E_INVALID, "null config");
  if (c->weight_dtype != 1 && c->weight_dtype != 3)
    return set_error(YB_E_UNSUPPORTED, "weights must be fp16 (dtype F16) or fp8 E5M2 (dtype F8_E5M2)");
  if (c->n_experts != 0) return set_error(YB_E_UNSUPPORTED, "mixture-of-experts checkpoints are not supported");
  if (c->dim <= 0 || c->hidden_dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
      c->vocab_size <= 0 || c->max_seq_len <= 2)
    return set_error(YB_E_INVALID, "non-positive dimension in config");
  if (c->head_dim != 64 && c->head_dim != 128) return set_error(YB_E_UNSUPPORTED, "head_dim must be 64 or 128");
  if (c->n_heads % c->n_kv_heads) return set_error(YB_E_INVALID, "n_heads must be a multiple of n_kv_heads");
  const int gq = c->n_heads / c->n_kv_heads;
  if (gq != 1 && gq != 2 && gq != 4 && gq != 8) return set_error(YB_E_UNSUPPORTED, "n_heads / n_kv_heads must be 1, 2, 4 or 8");
  if (c->rotary_dim < 0 || c->rotary_dim > c->head_dim || (c->rotary_dim & 1))
    return set_error(YB_E_INVALID, "rotary_dim must be even and <= head_dim");
  if (c->dim % 8 || c->hidden_dim % 8) return set_error(YB_E_UNSUPPORTED, "dim and hidden_dim must be multiples of 8");
  if (c->act != 0 && c->act != 1) return set_error(YB_E_INVALID, "act must be 0 (gelu) or 1 (silu)");
  const int cm = c->weight_dtype == 3 ? 16 : 8;  // weights per 16-byte chunk
  if (c->dim % cm || c->hidden_dim % cm || (c->n_heads * c->head_dim) % cm)
    return set_error(YB_E_UNSUPPORTED, "fp8 weights need dim and hidden_dim multiples of 16");
  if (tp_size < 1 || c->n_kv_heads % tp_size || c->hidden_dim % (cm * tp_size) || c->vocab_size % tp_size)
    return set_error(YB_E_INVALID, "tp_size must divide n_kv_heads, vocab_size and hidden_dim/8 (/16 for fp8)");
  return 0;
}


}  // namespace

// The slices of every tensor-parallel matrix that rank r of P holds (yb_tp_shard exports the same
// table): query heads (rows of Wq, columns of Wo) and kv heads (rows of Wk, Wv) in blocks of whole
// heads, so each GQA group stays on one rank; hidden units (rows of W1, W3, columns of W2); and
// classifier rows.  Element index ranges [begin, end).
static ShardTable shard_table(const yb_config& c, int r, int P) {
  const long long qr = (long long)(c.n_heads / P) * c.head_dim, kr = (long long)(c.n_kv_heads / P) * c.head_dim;
  const long long h = c.hidden_dim / P, v = c.vocab_size / P;
  return ShardTable{r * qr, (r + 1) * qr, r * kr, (r + 1) * kr, r * h, (r + 1) * h, r * v, (r + 1) * v};
}

static int upload_weights(yb_engine* e, const yb_weights* w) {
  const yb_config& c = e->cfg;
  const ShardTable& st = e->shard;
  const size_t dim = c.dim, hd = c.head_dim;
  const size_t q_dim = (size_t)c.n_heads * hd;
  const size_t es = e->esz;  // bytes per weight
  auto bytes = [](const void* p) { return static_cast<const unsigned char*>(p); };
  Loader ld;
  int rc;
  if ((rc = ld.init())) return rc;
  if ((rc = dev_alloc(e, &e->emb, (size_t)c.vocab_size * dim * es))) return rc;
  if ((rc = ld.contiguous(e->emb, w->token_embedding_table, (size_t)c.vocab_size * dim * es))) return rc;
  if ((rc = dev_alloc(e, &e->rms_final, dim * 4))) return rc;
  if ((rc = ld.contiguous(e->rms_final, w->rms_final_weight, dim * 4))) return rc;
  if (e->tp_size == 1 && w->wcls == w->token_embedding_table) {
    e->wcls = e->emb;  // tied embeddings
  } else {
    if ((rc = dev_alloc(e, &e->wcls, (size_t)e->vocab_l * dim * es))) return rc;
    if ((rc = ld.contiguous(e->wcls, bytes(w->wcls) + (size_t)st.v0 * dim * es, (size_t)e->vocab_l * dim * es)))
      return rc;
  }
  e->layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    LayerBuffers& L = e->layers[l];
    if (!w->wq[l] || !w->wk[l] || !w->wv[l] || !w->wo[l] || !w->w1[l] || !w->w2[l] || !w->w3[l] ||
        !w->rms_att_weight[l] || !w->rms_ffn_weight[l])
      return set_error(YB_E_INVALID, "missing tensor for layer " + std::to_string(l));
    if ((rc = dev_alloc(e, &L.rms_att, dim * 4))) return rc;
    if ((rc = dev_alloc(e, &L.rms_ffn, dim * 4))) return rc;
    if ((rc = ld.contiguous(L.rms_att, w->rms_att_weight[l], dim * 4))) return rc;
    if ((rc = ld.contiguous(L.rms_ffn, w->rms_ffn_weight[l], dim * 4))) return rc;
    // [Wq rows of this rank's heads; Wk rows; Wv rows]
    const size_t qr = e->q_rows, kr = e->kv_rows;
    if ((rc = dev_alloc(e, &L.wqkv, (qr + 2 * kr) * dim * es))) return rc;
    const unsigned char* wq = bytes(w->wq[l]) + (size_t)st.q0 * dim * es;
    const unsigned char* wk = bytes(w->wk[l]) + (size_t)st.kv0 * dim * es;
    const unsigned char* wv = bytes(w->wv[l]) + (size_t)st.kv0 * dim * es;
    const size_t rb = dim * es;  // bytes per row of a dim-wide matrix
    rc = ld.rows(L.wqkv, qr + 2 * kr, rb, [=](size_t i) -> const void* {
      return i < qr ? wq + i * rb : i < qr + kr ? wk + (i - qr) * rb : wv + (i - qr - kr) * rb;
    });
    if (rc) return rc;
    // Wo columns of this rank's heads
    if ((rc = dev_alloc(e, &L.wo, dim * qr * es))) return rc;
    const unsigned char* wo = bytes(w->wo[l]) + (size_t)st.q0 * es;
    if ((rc = ld.rows(L.wo, dim, qr * es, [=](size_t i) -> const void* { return wo + i * q_dim * es; }))) return rc;
    // W1 / W3 rows of this rank's hidden slice, interleaved (row 2i = W1 row i, 2i+1 = W3 row i)
    const size_t h = e->hid;
    if ((rc = dev_alloc(e, &L.w13, 2 * h * dim * es))) return rc;
    const unsigned char* w1 = bytes(w->w1[l]) + (size_t)st.h0 * rb;
    const unsigned char* w3 = bytes(w->w3[l]) + (size_t)st.h0 * rb;
    rc = ld.rows(L.w13, 2 * h, rb, [=](size_t i) -> const void* { return ((i & 1) ? w3 : w1) + (i >> 1) * rb; });
    if (rc) return rc;
    // W2 columns of the hidden slice
    if ((rc = dev_alloc(e, &L.w2, dim * h * es))) return rc;
    const unsigned char* w2 = bytes(w->w2[l]) + (size_t)st.h0 * es;
    const size_t hid_row = (size_t)c.hidden_dim * es;
    if ((rc = ld.rows(L.w2, dim, h * es, [=](size_t i) -> const void* { return w2 + i * hid_row; }))) return rc;
    // KV cache, zero-initialised like yalm's (src/model.cpp:203-204)
    const size_t kvb = (size_t)e->nkv * c.max_seq_len * hd * 2;
    if ((rc = dev_alloc(e, &L.k_cache, kvb))) return rc;
    if ((rc = dev_alloc(e, &L.v_cache, kvb))) return rc;
    YB_CK(cudaMemset(L.k_cache, 0, kvb));
    YB_CK(cudaMemset(L.v_cache, 0, kvb));
    if (!attn_maps(&L.attn_maps, L.k_cache, L.v_cache, e->nkv, c.max_seq_len, hd))
      return set_error(YB_E_CUDA, "tensor map encoding of the KV cache failed");
  }
  if ((rc = ld.finish())) return rc;
  e->upload_bytes = ld.bytes();
  if (e->esz == 1 && e->tune.fp8_mma) {
    // the tensor-core fp8 matvec reads 16-row groups (fp8_group_layout): re-lay each matrix into a
    // new buffer and release the row-major one (the embedding table stays row-major for the step
    // kernel; a classifier tied to it gets its own grouped copy)
    auto regroup = [&](__half** p, size_t rows, size_t cols, bool release) -> int {
      __half* nb = nullptr;
      int r = dev_alloc(e, &nb, fp8_group_bytes((long long)rows, (int)cols));
      if (r) return r;
      YB_CK(fp8_group_layout(*p, nb, (long long)rows, (int)cols, nullptr));
      YB_CK(cudaDeviceSynchronize());
      if (release) {
        for (size_t i = 0; i < e->allocs.size(); ++i)
          if (e->allocs[i] == *p) {
            e->allocs.erase(e->allocs.begin() + (long)i);
            YB_CK(cudaFree(*p));
            break;
          }
      }
      *p = nb;
      return 0;
    };
    for (int l = 0; l < c.n_layers; ++l) {
      LayerBuffers& L = e->layers[l];
      if ((rc = regroup(&L.wqkv, (size_t)e->q_rows + 2 * e->kv_rows, dim, true))) return rc;
      if ((rc = regroup(&L.wo, dim, (size_t)e->q_rows, true))) return rc;
      if ((rc = regroup(&L.w13, 2 * (size_t)e->hid, dim, true))) return rc;
      if ((rc = regroup(&L.w2, dim, (size_t)e->hid, true))) return rc;
    }
    if ((rc = regroup(&e->wcls, (size_t)e->vocab_l, dim, e->wcls != e->emb))) return rc;
    e->fp8_grouped = true;
  }
  return 0;
}

// This rank's exchange words of point pt (all ranks' partials, [tp][dim]).
static const unsigned long long* tp_in(yb_engine* e, int pt) {
  return reinterpret_cast<const unsigned long long*>(static_cast<char*>(e->tp.base) + e->tp.x_off) +
         (size_t)pt * e->tp_size * e->cfg.dim;
}

// Matrix pointer `cols` weights into each row (a column panel), for either weight type.
static const __half* wcols(const yb_engine* e, const __half* base, size_t cols) {
  // grouped fp8 (fp8_group_layout): a panel starts `cols` 16-row columns, cols * 16 bytes, in
  return reinterpret_cast<const __half*>(reinterpret_cast<const unsigned char*>(base) +
                                         cols * (e->fp8_grouped ? 16 : e->esz));
}

static GemvArgs base_args(yb_engine* e) {
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  a.status = e->status_d;
  a.step = e->step;
  a.eps = e->cfg.norm_eps;
  a.tp_size = e->tp_size;
  return a;
}

// The sampler after the classifier: one CTA over the logits every rank holds.
static int launch_sampler(yb_engine* e, cudaStream_t s, const StepState* step, SampleParams direct) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kSampleThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  YB_CK(cudaLaunchKernelEx(&cfg, sample_kernel, yb_logits_dev(e), e->cfg.vocab_size, step, direct, e->sample_d));
  return 0;
}

int record_step(yb_engine* e, int mode, const StepArgs& sa) {
  const yb_config& c = e->cfg;
  cudaStream_t s = e->stream;
  {
    StepArgs a = sa;
    YB_CK(launch_kernel(reinterpret_cast<const void*>(&step_kernel), dim3(4), dim3(1024), 0, s, false, &a));
  }
  const bool tp = e->tp_size > 1;
  const int pf = e->tune.l2_prefetch_stages;
  float* x_cur = e->x;  // TP: the residual stream ping-pongs between x and x2
  int kix = 0;          // kernel index within the step (timeline column block)
  auto timeline = [&](unsigned long long** tr, int* stride) {
    *tr = e->gtrace ? e->gtrace + (size_t)kix * 8 : nullptr;
    *stride = e->gtrace_events;
    ++kix;
  };
  for (int l = 0; l < c.n_layers; ++l) {
    LayerBuffers& L = e->layers[l];
    // ---- QKV
    {
      GemvArgs a = base_args(e);
      a.w = L.wqkv;
      a.ldw = c.dim;
      a.rows = e->q_rows + 2 * e->kv_rows;
      a.cols = c.dim;
      a.x = x_cur;
      a.norm_w = L.rms_att;
      a.y = e->q;
      a.q_rows = e->q_rows;
      a.kv_rows = e->kv_rows;
      a.head_dim = c.head_dim;
      a.rotary_dim = c.rotary_dim;
      a.max_seq_len = c.max_seq_len;
      a.qkv_clip = c.qkv_clip;
      a.inv_freq = e->inv_freq;
      a.k_cache = L.k_cache;
      a.v_cache = L.v_cache;
      a.kv_prefetch = 1;
      if (tp && l > 0) {
        // add the previous layer's w2 partials (exchange point 2l-1)
        a.tp_ll = tp_in(e, 2 * l - 1);
        a.tp_bar = e->tp.d_bar + (2 * l - 1);
        float* x_next = (x_cur == e->x) ? e->x2 : e->x;
        a.x_out = x_next;
        x_cur = x_next;
      }
      if (e->tune.prefetch_wo) {
        a.pf_src = reinterpret_cast<const unsigned char*>(L.wo);
        a.pf_bytes = (long long)c.dim * e->q_rows * e->esz;
      }
      timeline(&a.trace, &a.trace_stride);
      YB_CK(gemv_launch(a.tp_ll ? e->plan_qkv_tp : e->plan_qkv, a, s, true,
                        e->tune.l2_prefetch_qkv >= 0 ? e->tune.l2_prefetch_qkv : pf));
    }
    // ---- attention
    {
      AttnArgs a;
      std::memset(&a, 0, sizeof(a));
      a.q = e->q;
      a.k_cache = L.k_cache;
      a.v_cache = L.v_cache;
      a.out = e->att;
      a.part = e->attn_part;
      a.counters = e->attn_cnt;
      a.step = e->step;
      a.max_seq_len = c.max_seq_len;
      a.cta_slots = e->tune.attn_cta_slots;
      a.cluster_slots = e->tune.attn_cluster_slots;
      a.status = e->status_d;
      timeline(&a.trace, &a.trace_stride);
      YB_CK(attn_launch(e->plan_attn, a, L.attn_maps, s, true));
    }
    // ---- wo (+ residual, or partials to peers)
    {
      GemvArgs a = base_args(e);
      a.w = L.wo;
      a.ldw = e->q_rows;
      a.rows = c.dim;
      a.cols = e->q_rows;
      a.x = e->att;
      if (tp) {
        a.peer_ll = e->tp.d_peer_ll + (size_t)(2 * l) * e->tp_size;
      } else {
        a.y = x_cur;
      }
      timeline(&a.trace, &a.trace_stride);
      YB_CK(gemv_launch(e->plan_wo, a, s, true, e->tune.l2_prefetch_wo >= 0 ? e->tune.l2_prefetch_wo : pf));
    }
    // ---- gate/up (+ RMSNorm, SwiGLU)
    {
      GemvArgs a = base_args(e);
      a.w = L.w13;
      a.ldw = c.dim;
      a.rows = 2 * e->hid;
      a.cols = c.dim;
      a.x = x_cur;
      a.norm_w = L.rms_ffn;
      a.y = e->hb;
      a.act_silu = c.act;
      if (tp) {
        a.tp_ll = tp_in(e, 2 * l);
        a.tp_bar = e->tp.d_bar + 2 * l;
        float* x_next = (x_cur == e->x) ? e->x2 : e->x;
        a.x_out = x_next;
        x_cur = x_next;
      }
      timeline(&a.trace, &a.trace_stride);
      YB_CK(gemv_launch(e->plan_gu, a, s, true, pf));
    }
    // ---- w2 (+ residual, or partials to peers); column panels when hidden_l > 14336
    {
      const int panels = e->w2_panels;
      const int pcols = e->hid / panels;
      for (int p = 0; p < panels; ++p) {
        GemvArgs a = base_args(e);
        a.w = wcols(e, L.w2, (size_t)p * pcols);
        a.ldw = e->hid;
        a.rows = c.dim;
        a.cols = pcols;
        a.x = e->hb + (size_t)p * pcols;
        if (tp) {
          a.peer_ll = e->tp.d_peer_ll + (size_t)(2 * l + 1) * e->tp_size;
        } else {
          a.y = x_cur;
        }
        if (e->tune.prefetch_qkv && p == panels - 1 && l + 1 < c.n_layers) {
          a.pf_src = reinterpret_cast<const unsigned char*>(e->layers[l + 1].wqkv);
          a.pf_bytes = (long long)(e->q_rows + 2 * e->kv_rows) * c.dim * e->esz;
        }
        timeline(&a.trace, &a.trace_stride);
        YB_CK(gemv_launch(e->plan_w2, a, s, true, pf));
      }
    }
  }
  if (mode != kStepHydrate) {
    GemvArgs a = base_args(e);
    a.w = e->wcls;
    a.ldw = c.dim;
    a.rows = e->vocab_l;
    a.cols = c.dim;
    a.x = x_cur;
    a.norm_w = e->rms_final;
    if (tp) {
      a.tp_ll = tp_in(e, 2 * c.n_layers - 1);
      a.tp_bar = e->tp.d_bar + (2 * c.n_layers - 1);
      a.x_out = (x_cur == e->x) ? e->x2 : e->x;  // the final x, formed share by share
      a.peer_slots = e->tp.d_peer_slots;
      a.peer_counters = e->tp.d_peer_counters;
      a.row_offset = e->tp_rank * e->vocab_l;
    } else {
      a.y = e->logits;
    }
    timeline(&a.trace, &a.trace_stride);
    YB_CK(gemv_launch(e->plan_cls, a, s, true, pf));
    if (tp) {
      const unsigned* cnt = reinterpret_cast<const unsigned*>(static_cast<char*>(e->tp.base) + e->tp.cnt_off);
      struct {
        const StepState* step;
        const unsigned* counters;
        int tp_size;
        int grid;
        unsigned* status;
      } wa = {e->step, cnt, e->tp_size, e->plan_cls.grid, e->status_d};
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1);
      cfg.blockDim = dim3(32);
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      YB_CK(cudaLaunchKernelEx(&cfg, tp_gather_wait_kernel, wa.step, wa.counters, wa.tp_size, wa.grid, wa.status));
    }
    if (mode == kStepSample) {
      const int rc = launch_sampler(e, s, e->step, SampleParams{});
      if (rc) return rc;
    }
  }
  return 0;
}

static int build_graph(yb_engine* e, int mode) {
  StepArgs sa{e->step, e->x, e->emb, e->cfg.dim, 0, 0, e->cfg.max_seq_len, 0, 0, 0, 0, 0.f, 0.f,
              e->tp.d_bar, e->tp.d_bar ? 2 * e->cfg.n_layers : 0, e->esz};
  cudaGraph_t g = nullptr;
  YB_CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  int rc = record_step(e, mode, sa);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return set_error(YB_E_CUDA, std::string("cudaStreamEndCapture: ") + cudaGetErrorString(ce));
  size_t n_roots = 0;
  YB_CK(cudaGraphGetRootNodes(g, nullptr, &n_roots));
  if (n_roots != 1) {
    cudaGraphDestroy(g);
    return set_error(YB_E_CUDA, "unexpected graph shape: " + std::to_string(n_roots) + " root nodes");
  }
  cudaGraphNode_t root;
  YB_CK(cudaGraphGetRootNodes(g, &root, &n_roots));
  e->step_node[mode] = root;
  // the graph stays alive: the step node handle used for per-call parameter updates belongs to it
  e->graph[mode] = g;
  cudaError_t ie = cudaGraphInstantiate(&e->exec[mode], g, 0);
  if (ie != cudaSuccess) return set_error(YB_E_CUDA, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(ie));
  return 0;
}

}  // namespace yb

using namespace yb;

static int engine_init(yb_engine* e, const yb_config* cfg, const yb_weights* w, int device, int tp_rank, int tp_size) {
  int rc = check_config(cfg, tp_size);
  if (rc) return rc;
  if (!w) return set_error(YB_E_INVALID, "null weights");
  if (tp_rank < 0 || tp_rank >= tp_size) return set_error(YB_E_INVALID, "tp_rank out of range");
  e->cfg = *cfg;
  e->esz = cfg->weight_dtype == 3 ? 1 : 2;
  e->tune = LaunchTuning::from_env();
  e->device = device;
  e->tp_rank = tp_rank;
  e->tp_size = tp_size;
  const yb_config& c = e->cfg;
  e->shard = shard_table(c, tp_rank, tp_size);
  e->nh = c.n_heads / tp_size;
  e->nkv = c.n_kv_heads / tp_size;
  e->q_rows = (int)(e->shard.q1 - e->shard.q0);
  e->kv_rows = (int)(e->shard.kv1 - e->shard.kv0);
  e->hid = (int)(e->shard.h1 - e->shard.h0);
  e->vocab_l = (int)(e->shard.v1 - e->shard.v0);
  YB_CK(cudaSetDevice(device));
  YB_CK(cudaDeviceGetAttribute(&e->n_sms, cudaDevAttrMultiProcessorCount, device));
  YB_CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  YB_CK(cudaHostAlloc(reinterpret_cast<void**>(&e->status_h), 64, cudaHostAllocMapped));
  std::memset(e->status_h, 0, 64);
  YB_CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->status_d), e->status_h, 0));
  YB_CK(cudaHostAlloc(reinterpret_cast<void**>(&e->sample_h), sizeof(SampleResult), cudaHostAllocMapped));
  std::memset(e->sample_h, 0, sizeof(SampleResult));
  YB_CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->sample_d), e->sample_h, 0));

  if ((rc = upload_weights(e, w))) return rc;

  // RoPE frequencies exactly as yalm computes them: 1 / powf(theta, j / rotary_dim) for even j
  // (src/infer.cpp:205), here once on the host.
  std::vector<float> inv(c.head_dim / 2, 0.f);
  for (int j = 0; j < c.head_dim; j += 2)
    inv[j / 2] = j >= c.rotary_dim ? 0.f : 1.0f / powf(c.rope_theta, (float)j / (float)c.rotary_dim);
  if ((rc = dev_alloc(e, &e->inv_freq, inv.size() * 4))) return rc;
  YB_CK(cudaMemcpy(e->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice));

  if ((rc = dev_alloc(e, &e->x, (size_t)c.dim * 4))) return rc;
  if ((rc = dev_alloc(e, &e->x2, (size_t)c.dim * 4))) return rc;
  if ((rc = dev_alloc(e, &e->q, (size_t)e->q_rows * 4))) return rc;
  if ((rc = dev_alloc(e, &e->att, (size_t)e->q_rows * 4))) return rc;
  if ((rc = dev_alloc(e, &e->hb, (size_t)e->hid * 4))) return rc;
  if ((rc = dev_alloc(e, &e->logits, (size_t)c.vocab_size * 4))) return rc;
  if ((rc = dev_alloc(e, &e->step, sizeof(StepState)))) return rc;
  YB_CK(cudaMemset(e->x, 0, (size_t)c.dim * 4));
  YB_CK(cudaMemset(e->x2, 0, (size_t)c.dim * 4));
  YB_CK(cudaMemset(e->step, 0, sizeof(StepState)));

  // kernel plans
  const int epi_res = tp_size > 1 ? kEpiResidTP : kEpiResid;
  e->plan_qkv = gemv_plan(e->q_rows + 2 * e->kv_rows, c.dim, kEpiQKV, true, e->n_sms, e->tune, false, e->esz);
  e->plan_wo = gemv_plan(c.dim, e->q_rows, epi_res, false, e->n_sms, e->tune, false, e->esz);
  e->plan_gu = gemv_plan(2 * e->hid, c.dim, kEpiGateUp, true, e->n_sms, e->tune, tp_size > 1, e->esz);
  e->plan_qkv_tp = tp_size > 1 ? gemv_plan(e->q_rows + 2 * e->kv_rows, c.dim, kEpiQKV, true, e->n_sms, e->tune, true, e->esz)
                               : e->plan_qkv;
  e->w2_panels = 1;
  const int col_mult = e->esz == 1 ? 16 : 8;  // columns per 16-byte chunk
  while (gemv_kpt_for(e->hid / e->w2_panels, e->esz) < 0 || (e->hid / e->w2_panels) % col_mult || e->hid % e->w2_panels) {
    if (++e->w2_panels > 16) return set_error(YB_E_UNSUPPORTED, "hidden_dim too large");
  }
  if (tp_size > 1 && e->w2_panels > 1) return set_error(YB_E_UNSUPPORTED, "hidden_dim per rank too large for tensor parallelism");
  e->plan_w2 = gemv_plan(c.dim, e->hid / e->w2_panels, epi_res, false, e->n_sms, e->tune, false, e->esz);
  e->plan_cls = gemv_plan(e->vocab_l, c.dim, tp_size > 1 ? kEpiStoreTP : kEpiStore, true, e->n_sms, e->tune, tp_size > 1, e->esz);
  e->plan_attn = attn_plan(e->nh, e->nkv, c.head_dim, c.max_seq_len);
  if (!e->plan_qkv.ok || !e->plan_qkv_tp.ok || !e->plan_wo.ok || !e->plan_gu.ok || !e->plan_w2.ok ||
      !e->plan_cls.ok || !e->plan_attn.ok)
    return set_error(YB_E_UNSUPPORTED, "no kernel configuration for this model shape");
  for (const GemvPlan* p : {&e->plan_qkv, &e->plan_qkv_tp, &e->plan_wo, &e->plan_gu, &e->plan_w2, &e->plan_cls})
    YB_CK(gemv_prepare(*p));
  YB_CK(attn_prepare(e->plan_attn));
  // persistent executor: one cooperative kernel per step when an instantiation fits this shape
  {
    const char* ex = std::getenv("YB_EXECUTOR");
    const bool want = ex && std::string(ex) == "persistent";
    int coop = 0;
    YB_CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
    if (want && coop && tp_size == 1 && e->esz == 2) {
      PersistPlan pp = persist_plan(c.dim, e->q_rows, e->hid, c.head_dim, c.n_heads / c.n_kv_heads, e->n_sms);
      if (pp.ok) {
        const int G = pp.grid;
        int red = 0, max_local = 0;
        const int shapes[5][2] = {{e->q_rows + 2 * e->kv_rows, pp.rd}, {c.dim, pp.ro}, {2 * e->hid, pp.rd},
                                  {c.dim, pp.rh}, {e->vocab_l, pp.rd}};
        for (auto& sh : shapes) {
          const int ml = persist_max_local(sh[0], sh[1], G, e->tune.persist_static_pct);
          max_local = std::max(max_local, ml);
          red = std::max(red, ml * sh[1] * kPWarps);
        }
        YB_CK(persist_prepare(pp));
        int per_sm = 0;
        const size_t smem = persist_smem_bytes(red, max_local);
        YB_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pp.fn, kPThreads, smem));
        if (per_sm >= 1) {
          e->persistent = true;
          e->plan_persist = pp;
          e->persist_red_floats = red;
          e->persist_max_local = max_local;
        }
      }
    }
  }
  if (e->persistent) {
    std::vector<PLayer> pl(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
      const LayerBuffers& L = e->layers[l];
      pl[l] = PLayer{L.wqkv, L.wo, L.w13, L.w2, L.rms_att, L.rms_ffn, L.k_cache, L.v_cache};
    }
    if ((rc = dev_alloc(e, &e->d_players, pl.size() * sizeof(PLayer)))) return rc;
    YB_CK(cudaMemcpy(e->d_players, pl.data(), pl.size() * sizeof(PLayer), cudaMemcpyHostToDevice));
    // barrier counter (8 B), failure flag (4 B), one stage-claim counter per phase (4 B each)
    e->persist_sync_bytes = (12 + 4 * (5 * (size_t)c.n_layers + 1) * e->tune.persist_claim_ctrs + 15) / 16 * 16;
    if ((rc = dev_alloc(e, &e->persist_sync, e->persist_sync_bytes))) return rc;
    YB_CK(cudaMemset(e->persist_sync, 0, e->persist_sync_bytes));
    const char* tr = std::getenv("YB_TRACE");
    if (tr && tr[0] == '1') {
      const size_t n = (size_t)e->plan_persist.grid * kTraceEvents;
      if ((rc = dev_alloc(e, &e->trace, n * 8))) return rc;
      YB_CK(cudaMemset(e->trace, 0, n * 8));
    }
  }
  {
    const size_t pf = std::max(e->plan_attn.part_floats, (size_t)e->nh * kPMaxSplits * (c.head_dim + 2));
    if ((rc = dev_alloc(e, &e->attn_part, pf * 4))) return rc;
  }
  if ((rc = dev_alloc(e, &e->attn_cnt, (size_t)e->nkv * 4))) return rc;
  YB_CK(cudaMemset(e->attn_cnt, 0, (size_t)e->nkv * 4));
  if (!e->persistent) {
    const char* tr = std::getenv("YB_TRACE");
    if (tr && tr[0] == '1') {
      int rows = (int)(e->plan_attn.grid.x * e->plan_attn.grid.y);
      for (const GemvPlan* p : {&e->plan_qkv, &e->plan_wo, &e->plan_gu, &e->plan_w2, &e->plan_cls})
        rows = std::max(rows, p->grid);
      const int n_kern = c.n_layers * (4 + e->w2_panels) + 1;
      e->gtrace_rows = rows;
      e->gtrace_events = n_kern * 8;
      const size_t n = (size_t)rows * e->gtrace_events;
      if ((rc = dev_alloc(e, &e->gtrace, n * 8))) return rc;
      YB_CK(cudaMemset(e->gtrace, 0, n * 8));
    }
  }

  if (tp_size > 1) {
    // exchange region: partial-sum slots, gathered logits, arrival counters
    TpRegion& t = e->tp;
    const size_t n_pts = 2 * (size_t)c.n_layers;
    t.x_off = 0;
    t.logit_off = n_pts * tp_size * c.dim * 8;
    t.cnt_off = t.logit_off + (size_t)c.vocab_size * 4;
    t.bytes = t.cnt_off + (size_t)tp_size * 4;
    t.bytes = (t.bytes + 4095) / 4096 * 4096;
    YB_CK(cudaMalloc(&t.base, t.bytes));
    YB_CK(cudaMemset(t.base, 0, t.bytes));
    // graphs are recorded in yb_tp_import once the peers are mapped
    YB_CK(cudaDeviceSynchronize());
    return 0;
  }
  if (!e->persistent) {
    for (int m = 0; m < kStepVariants; ++m)
      if ((rc = build_graph(e, m))) return rc;
  }
  YB_CK(cudaDeviceSynchronize());
  return 0;
}

extern "C" int yb_create(const yb_config* cfg, const yb_weights* w, int device, int tp_rank, int tp_size,
                         yb_engine** out) {
  if (!out) return set_error(YB_E_INVALID, "null output pointer");
  *out = nullptr;
  yb_engine* e = new yb_engine();
  int rc = engine_init(e, cfg, w, device, tp_rank, tp_size);
  if (rc) {
    std::string msg = last_error();
    yb_destroy(e);
    return set_error(rc, msg);
  }
  *out = e;
  return 0;
}

static int launch_step(yb_engine* e, int token, int pos, int mode, const SampleParams* sp = nullptr) {
  if (!e) return set_error(YB_E_INVALID, "null engine");
  if (mode != kStepHydrate && mode != kStepLogits && !(mode == kStepSample && sp))
    return set_error(YB_E_INVALID, "mode must be 0 (hydrate) or 1 (logits)");
  if (token < 0 || token >= e->cfg.vocab_size) return set_error(YB_E_INVALID, "token out of range");
  if (pos < 0) return set_error(YB_E_INVALID, "negative position");
  if (!e->persistent && !e->exec[mode])
    return set_error(YB_E_INVALID, "engine not ready (tensor-parallel engines need yb_tp_import)");
  YB_CK(cudaSetDevice(e->device));
  e->epoch += 1;
  if (mode != kStepHydrate) e->lepoch += 1;
  if (e->persistent) {
    const yb_config& c = e->cfg;
    PArgs a;
    std::memset(&a, 0, sizeof(a));
    a.layers = e->d_players;
    a.n_layers = c.n_layers;
    a.dim = c.dim;
    a.q_rows = e->q_rows;
    a.kv_rows = e->kv_rows;
    a.hid = e->hid;
    a.vocab_rows = e->vocab_l;
    a.head_dim = c.head_dim;
    a.rotary_dim = c.rotary_dim;
    a.max_seq_len = c.max_seq_len;
    a.n_kv = e->nkv;
    a.eps = c.norm_eps;
    a.qkv_clip = c.qkv_clip;
    a.act_silu = c.act;
    a.emb = e->emb;
    a.wcls = e->wcls;
    a.rms_final = e->rms_final;
    a.inv_freq = e->inv_freq;
    a.x = e->x;
    a.x2 = e->x2;
    a.q = e->q;
    a.att = e->att;
    a.hb = e->hb;
    a.logits = e->logits;
    a.attn_part = e->attn_part;
    a.attn_cnt = e->attn_cnt;
    a.bar = e->persist_sync;
    a.fail = reinterpret_cast<unsigned*>(e->persist_sync + 1);
    a.status = e->status_d;
    a.token = token;
    a.pos = pos;
    // src/infer.cpp:489-494
    a.kv_sink = pos >= c.max_seq_len ? 2 : 0;
    a.kv_pos = a.kv_sink + (pos - a.kv_sink) % (c.max_seq_len - a.kv_sink);
    a.kv_len = pos >= c.max_seq_len ? c.max_seq_len : pos + 1;
    a.mode = mode == kStepHydrate ? 0 : 1;
    a.epoch = e->epoch;
    a.lepoch = e->lepoch;
    a.tp_size = 1;
    a.red_floats = e->persist_red_floats;
    a.max_local = e->persist_max_local;
    a.static_pct = e->tune.persist_static_pct;
    a.claim_ctrs = e->tune.persist_claim_ctrs;
    a.trace = e->trace;
    YB_CK(cudaMemsetAsync(e->persist_sync, 0, e->persist_sync_bytes, e->stream));
    YB_CK(persist_launch(e->plan_persist, a, e->stream));
    if (mode == kStepSample) {
      SampleParams d = *sp;
      d.epoch = e->epoch;
      return launch_sampler(e, e->stream, nullptr, d);
    }
    return 0;
  }
  StepArgs sa{e->step, e->x, e->emb, e->cfg.dim, token, pos, e->cfg.max_seq_len, e->epoch, e->lepoch,
              sp ? sp->op : 0, sp ? sp->target : 0, sp ? sp->temperature : 0.f, sp ? sp->coin : 0.f,
              e->tp.d_bar, e->tp.d_bar ? 2 * e->cfg.n_layers : 0, e->esz};
  cudaKernelNodeParams kp = {};
  void* params[] = {&sa};
  kp.func = reinterpret_cast<void*>(&step_kernel);
  kp.gridDim = dim3(4);
  kp.blockDim = dim3(1024);
  kp.sharedMemBytes = 0;
  kp.kernelParams = params;
  YB_CK(cudaGraphExecKernelNodeSetParams(e->exec[mode], e->step_node[mode], &kp));
  YB_CK(cudaGraphLaunch(e->exec[mode], e->stream));
  return 0;
}

static int check_status(yb_engine* e) {
  const unsigned st = *reinterpret_cast<volatile unsigned*>(e->status_h);
  if (st) {
    char buf[160];
    std::snprintf(buf, sizeof(buf),
                  "device status 0x%x (1: TMA stage wait, 2: peer wait, 8: grid barrier wait timed out; 4: bad args)", st);
    return set_error(YB_E_TIMEOUT, buf);
  }
  return 0;
}

extern "C" int yb_forward(yb_engine* e, int token, int pos, int mode, float* logits) {
  int rc = launch_step(e, token, pos, mode);
  if (rc) return rc;
  if (mode == YB_MODE_OUTPUT_LOGITS) {
    if (logits)
      YB_CK(cudaMemcpyAsync(logits, yb_logits_dev(e), (size_t)e->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, e->stream));
    YB_CK(cudaStreamSynchronize(e->stream));
    return check_status(e);
  }
  return 0;
}

extern "C" int yb_forward_async(yb_engine* e, int token, int pos, int mode) { return launch_step(e, token, pos, mode); }

static int forward_sampled(yb_engine* e, int token, int pos, const SampleParams& sp, SampleResult* res) {
  int rc = launch_step(e, token, pos, kStepSample, &sp);
  if (rc) return rc;
  YB_CK(cudaStreamSynchronize(e->stream));
  if ((rc = check_status(e))) return rc;
  const volatile SampleResult* v = e->sample_h;
  res->token = v->token;
  res->prob = v->prob;
  res->epoch = v->epoch;
  if (res->epoch != e->epoch) return set_error(YB_E_CUDA, "sampler result missing");
  return 0;
}

extern "C" int yb_forward_sample(yb_engine* e, int token, int pos, float temperature, float coin, int* next_token) {
  if (!next_token) return set_error(YB_E_INVALID, "null output pointer");
  if (!(temperature >= 0.f)) return set_error(YB_E_INVALID, "temperature must be >= 0");
  SampleParams sp{temperature == 0.f ? 0 : 1, 0, temperature, coin, 0};
  SampleResult r;
  int rc = forward_sampled(e, token, pos, sp, &r);
  if (rc) return rc;
  *next_token = r.token;
  return 0;
}

extern "C" int yb_forward_prob(yb_engine* e, int token, int pos, int target, float* prob) {
  if (!prob) return set_error(YB_E_INVALID, "null output pointer");
  if (!e || target < 0 || target >= e->cfg.vocab_size) return set_error(YB_E_INVALID, "target out of range");
  SampleParams sp{2, target, 1.f, 0.f, 0};
  SampleResult r;
  int rc = forward_sampled(e, token, pos, sp, &r);
  if (rc) return rc;
  *prob = r.prob;
  return 0;
}

extern "C" int yb_sync(yb_engine* e) {
  if (!e) return set_error(YB_E_INVALID, "null engine");
  YB_CK(cudaSetDevice(e->device));
  YB_CK(cudaStreamSynchronize(e->stream));
  return check_status(e);
}

extern "C" const float* yb_logits_dev(yb_engine* e) {
  if (!e) return nullptr;
  return e->tp_size > 1 ? reinterpret_cast<const float*>(static_cast<char*>(e->tp.base) + e->tp.logit_off) : e->logits;
}

extern "C" void* yb_stream(yb_engine* e) { return e ? static_cast<void*>(e->stream) : nullptr; }

extern "C" int yb_read_kv(yb_engine* e, int layer, int kv_head, int slot0, int n, uint16_t* k_out, uint16_t* v_out) {
  if (!e) return set_error(YB_E_INVALID, "null engine");
  if (layer < 0 || layer >= e->cfg.n_layers || kv_head < 0 || kv_head >= e->nkv || slot0 < 0 || n < 0 ||
      slot0 + n > e->cfg.max_seq_len)
    return set_error(YB_E_INVALID, "read_kv range out of bounds");
  YB_CK(cudaSetDevice(e->device));
  YB_CK(cudaStreamSynchronize(e->stream));
  const size_t hd = e->cfg.head_dim;
  const size_t off = ((size_t)kv_head * e->cfg.max_seq_len + slot0) * hd;
  if (k_out) YB_CK(cudaMemcpy(k_out, e->layers[layer].k_cache + off, (size_t)n * hd * 2, cudaMemcpyDeviceToHost));
  if (v_out) YB_CK(cudaMemcpy(v_out, e->layers[layer].v_cache + off, (size_t)n * hd * 2, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int yb_tp_shard(const yb_config* cfg, int tp_rank, int tp_size, long long* out8) {
  if (!cfg || !out8) return set_error(YB_E_INVALID, "null argument");
  int rc = check_config(cfg, tp_size);
  if (rc) return rc;
  if (tp_rank < 0 || tp_rank >= tp_size) return set_error(YB_E_INVALID, "tp_rank out of range");
  const ShardTable st = shard_table(*cfg, tp_rank, tp_size);
  const long long v[8] = {st.q0, st.q1, st.kv0, st.kv1, st.h0, st.h1, st.v0, st.v1};
  for (int i = 0; i < 8; ++i) out8[i] = v[i];
  return 0;
}

extern "C" int yb_executor(yb_engine* e) { return e && e->persistent ? 1 : 0; }

extern "C" int yb_trace_read(yb_engine* e, unsigned long long* out, size_t n, int* grid, int* events) {
  if (e && !e->persistent && e->gtrace) {
    const size_t total = (size_t)e->gtrace_rows * e->gtrace_events;
    if (grid) *grid = e->gtrace_rows;
    if (events) *events = e->gtrace_events;
    if (!out) return 0;
    if (n < total) return set_error(YB_E_INVALID, "timeline buffer too small");
    YB_CK(cudaSetDevice(e->device));
    YB_CK(cudaStreamSynchronize(e->stream));
    YB_CK(cudaMemcpy(out, e->gtrace, total * 8, cudaMemcpyDeviceToHost));
    return 0;
  }
  if (!e || !e->persistent || !e->trace) return set_error(YB_E_INVALID, "no timeline (engine created without YB_TRACE=1)");
  const size_t total = (size_t)e->plan_persist.grid * kTraceEvents;
  if (grid) *grid = e->plan_persist.grid;
  if (events) *events = kTraceEvents;
  if (!out) return 0;
  if (n < total) return set_error(YB_E_INVALID, "timeline buffer too small");
  YB_CK(cudaSetDevice(e->device));
  YB_CK(cudaStreamSynchronize(e->stream));
  YB_CK(cudaMemcpy(out, e->trace, total * 8, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" unsigned yb_status(yb_engine* e) { return e ? *reinterpret_cast<volatile unsigned*>(e->status_h) : 0u; }

extern "C" int yb_clear_status(yb_engine* e) {
  if (!e) return set_error(YB_E_INVALID, "null engine");
  *reinterpret_cast<volatile unsigned*>(e->status_h) = 0u;
  return 0;
}

extern "C" void yb_destroy(yb_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (int m = 0; m < kStepVariants; ++m) {
    if (e->exec[m]) cudaGraphExecDestroy(e->exec[m]);
    if (e->graph[m]) cudaGraphDestroy(e->graph[m]);
  }
  for (size_t i = 0; i < e->tp.peer_base.size(); ++i)
    if ((int)i != e->tp_rank && e->tp.peer_base[i]) cudaIpcCloseMemHandle(e->tp.peer_base[i]);
  if (e->tp.d_peer_ll) cudaFree(e->tp.d_peer_ll);
  if (e->tp.d_bar) cudaFree(e->tp.d_bar);
  if (e->tp.d_peer_slots) cudaFree(e->tp.d_peer_slots);
  if (e->tp.d_peer_counters) cudaFree(e->tp.d_peer_counters);
  if (e->tp.base) cudaFree(e->tp.base);
  for (void* p : e->allocs) cudaFree(p);
  for (void* v : {(void*)e->pf.x, (void*)e->pf.xn, (void*)e->pf.qkv, (void*)e->pf.q, (void*)e->pf.att, (void*)e->pf.h,
                  (void*)e->pf.tokens})
    if (v) cudaFree(v);
  if (e->status_h) cudaFreeHost(e->status_h);
  if (e->sample_h) cudaFreeHost(e->sample_h);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

extern "C" int yb_profile_kernel(yb_engine* e, int which, int iters, float* ms_per_launch) {
  if (!e || !ms_per_launch || iters <= 0 || which < 0 || which > 5) return set_error(YB_E_INVALID, "bad profile arguments");
  if (e->tp_size > 1) return set_error(YB_E_INVALID, "profiling is for single-GPU engines");
  YB_CK(cudaSetDevice(e->device));
  const yb_config& c = e->cfg;
  cudaEvent_t a, b;
  YB_CK(cudaEventCreate(&a));
  YB_CK(cudaEventCreate(&b));
  int rc = 0;
  auto one = [&](int i) -> int {
    const int l = i % c.n_layers;
    LayerBuffers& L = e->layers[l];
    const int pf = e->tune.l2_prefetch_stages;
    GemvArgs g = base_args(e);
    switch (which) {
      case 0:
        g.w = L.wqkv; g.ldw = c.dim; g.rows = e->q_rows + 2 * e->kv_rows; g.cols = c.dim; g.x = e->x;
        g.norm_w = L.rms_att; g.y = e->q; g.q_rows = e->q_rows; g.kv_rows = e->kv_rows; g.head_dim = c.head_dim;
        g.rotary_dim = c.rotary_dim; g.max_seq_len = c.max_seq_len; g.qkv_clip = c.qkv_clip; g.inv_freq = e->inv_freq;
        g.k_cache = L.k_cache; g.v_cache = L.v_cache;
        YB_CK(gemv_launch(e->plan_qkv, g, e->stream, true, pf));
        return 0;
      case 1: {
        AttnArgs t;
        std::memset(&t, 0, sizeof(t));
        t.q = e->q; t.k_cache = L.k_cache; t.v_cache = L.v_cache; t.out = e->att; t.part = e->attn_part;
        t.counters = e->attn_cnt; t.step = e->step; t.max_seq_len = c.max_seq_len; t.status = e->status_d;
        t.cta_slots = e->tune.attn_cta_slots;
        t.cluster_slots = e->tune.attn_cluster_slots;
        YB_CK(attn_launch(e->plan_attn, t, L.attn_maps, e->stream, true));
        return 0;
      }
      case 2:
        g.w = L.wo; g.ldw = e->q_rows; g.rows = c.dim; g.cols = e->q_rows; g.x = e->att; g.y = e->x;
        YB_CK(gemv_launch(e->plan_wo, g, e->stream, true, pf));
        return 0;
      case 3:
        g.w = L.w13; g.ldw = c.dim; g.rows = 2 * e->hid; g.cols = c.dim; g.x = e->x; g.norm_w = L.rms_ffn;
        g.y = e->hb; g.act_silu = c.act;
        YB_CK(gemv_launch(e->plan_gu, g, e->stream, true, pf));
        return 0;
      case 4: {
        const int pcols = e->hid / e->w2_panels;
        for (int p = 0; p < e->w2_panels; ++p) {
          GemvArgs h = base_args(e);
          h.w = wcols(e, L.w2, (size_t)p * pcols); h.ldw = e->hid; h.rows = c.dim; h.cols = pcols;
          h.x = e->hb + (size_t)p * pcols; h.y = e->x;
          YB_CK(gemv_launch(e->plan_w2, h, e->stream, true, pf));
        }
        return 0;
      }
      default:
        g.w = e->wcls; g.ldw = c.dim; g.rows = e->vocab_l; g.cols = c.dim; g.x = e->x; g.norm_w = e->rms_final;
        g.y = e->logits;
        YB_CK(gemv_launch(e->plan_cls, g, e->stream, true, pf));
        return 0;
    }
  };
  // one untimed pass over every layer first (first-launch costs, L2 state comparable to a step)
  for (int i = 0; i < c.n_layers && !rc; ++i) rc = one(i);
  if (!rc) {
    cudaEventRecord(a, e->stream);
    for (int i = 0; i < iters && !rc; ++i) rc = one(i);
    cudaEventRecord(b, e->stream);
  }
  cudaError_t se = cudaEventSynchronize(b);
  float ms = 0.f;
  if (!rc && se == cudaSuccess) cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (rc) return rc;
  if (se != cudaSuccess) return set_error(YB_E_CUDA, std::string("profile: ") + cudaGetErrorString(se));
  *ms_per_launch = ms / (float)iters;
  return check_status(e);
}

extern "C" int yb_last_error(char* buf, int n) {
  const std::string& m = last_error();
  if (buf && n > 0) {
    std::snprintf(buf, (size_t)n, "%s", m.c_str());
  }
  return (int)m.size();
}

// ------------------------------------------------------------------------------ tensor parallelism
struct TpBlob {
  unsigned magic;
  int rank;
  int tp_size;
  int pad;
  size_t bytes;
  cudaIpcMemHandle_t handle;
};

extern "C" size_t yb_tp_blob_bytes(void) { return sizeof(TpBlob); }

extern "C" int yb_tp_export(yb_engine* e, void* blob, size_t blob_bytes, size_t* used) {
  if (!e || !blob) return set_error(YB_E_INVALID, "null argument");
  if (e->tp_size < 2) return set_error(YB_E_INVALID, "engine was not created for tensor parallelism");
  if (blob_bytes < sizeof(TpBlob)) return set_error(YB_E_INVALID, "blob buffer too small");
  YB_CK(cudaSetDevice(e->device));
  TpBlob b;
  std::memset(&b, 0, sizeof(b));
  b.magic = 0x59425450u;
  b.rank = e->tp_rank;
  b.tp_size = e->tp_size;
  b.bytes = e->tp.bytes;
  YB_CK(cudaIpcGetMemHandle(&b.handle, e->tp.base));
  std::memcpy(blob, &b, sizeof(b));
  if (used) *used = sizeof(b);
  return 0;
}

extern "C" int yb_tp_import(yb_engine* e, const void* blobs, size_t stride) {
  if (!e || !blobs) return set_error(YB_E_INVALID, "null argument");
  if (e->tp_size < 2) return set_error(YB_E_INVALID, "engine was not created for tensor parallelism");
  if (e->tp.joined) return set_error(YB_E_INVALID, "already joined");
  if (stride < sizeof(TpBlob)) return set_error(YB_E_INVALID, "blob stride too small");
  YB_CK(cudaSetDevice(e->device));
  const int P = e->tp_size;
  const yb_config& c = e->cfg;
  e->tp.peer_base.assign(P, nullptr);
  for (int r = 0; r < P; ++r) {
    TpBlob b;
    std::memcpy(&b, static_cast<const char*>(blobs) + (size_t)r * stride, sizeof(b));
    if (b.magic != 0x59425450u || b.rank != r || b.tp_size != P || b.bytes != e->tp.bytes)
      return set_error(YB_E_INVALID, "inconsistent tensor-parallel blob for rank " + std::to_string(r));
    if (r == e->tp_rank) {
      e->tp.peer_base[r] = e->tp.base;
    } else {
      void* p = nullptr;
      YB_CK(cudaIpcOpenMemHandle(&p, b.handle, cudaIpcMemLazyEnablePeerAccess));
      e->tp.peer_base[r] = p;
    }
  }
  // Destinations: at exchange point pt < 2L, rank `me` writes its partial words into rank p's
  // slot [pt][me][:]; the classifier writes its vocabulary rows into every rank's logits buffer and
  // bumps that rank's counter [me].
  const int n_pts = 2 * c.n_layers;
  std::vector<unsigned long long*> ll((size_t)n_pts * P);
  std::vector<float*> lg(P);
  std::vector<unsigned*> cnts(P);
  for (int p = 0; p < P; ++p) {
    char* base = static_cast<char*>(e->tp.peer_base[p]);
    for (int pt = 0; pt < n_pts; ++pt)
      ll[(size_t)pt * P + p] =
          reinterpret_cast<unsigned long long*>(base + e->tp.x_off) + ((size_t)pt * P + e->tp_rank) * c.dim;
    lg[p] = reinterpret_cast<float*>(base + e->tp.logit_off);
    cnts[p] = reinterpret_cast<unsigned*>(base + e->tp.cnt_off) + e->tp_rank;
  }
  YB_CK(cudaMalloc(&e->tp.d_peer_ll, ll.size() * sizeof(unsigned long long*)));
  YB_CK(cudaMalloc(&e->tp.d_bar, (size_t)n_pts * sizeof(unsigned)));
  YB_CK(cudaMemset(e->tp.d_bar, 0, (size_t)n_pts * sizeof(unsigned)));
  YB_CK(cudaMalloc(&e->tp.d_peer_slots, lg.size() * sizeof(float*)));
  YB_CK(cudaMalloc(&e->tp.d_peer_counters, cnts.size() * sizeof(unsigned*)));
  YB_CK(cudaMemcpy(e->tp.d_peer_ll, ll.data(), ll.size() * sizeof(unsigned long long*), cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(e->tp.d_peer_slots, lg.data(), lg.size() * sizeof(float*), cudaMemcpyHostToDevice));
  YB_CK(cudaMemcpy(e->tp.d_peer_counters, cnts.data(), cnts.size() * sizeof(unsigned*), cudaMemcpyHostToDevice));
  e->tp.joined = true;
  int rc;
  for (int m = 0; m < kStepVariants; ++m)
    if ((rc = build_graph(e, m))) return rc;
  YB_CK(cudaDeviceSynchronize());
  return 0;
}
