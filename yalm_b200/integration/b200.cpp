// yalm-side binding of the yalm_b200 engine: src/b200.cpp of a yalm checkout.
//
// Together with yalm.patch (a `-d b200` device: Model::cuda_b200() and a flag that Model::forward,
// src/model.cpp:479-494, checks first, and the device name in src/main.cpp) this file is everything
// yalm needs to run its completion, perplexity and passkey modes on the engine.  It fills the C
// ABI's structs (include/yalm_b200.h) from yalm's own Config / Block / Model objects before anything
// is uploaded — the tensor pointers are still the mmap'd .yalm data (src/model.cpp:392-435) — and
// forwards each Model::forward call to yb_forward, which writes the logits into the host buffer
// InferenceState::logits().  Model and InferenceState stay CPU objects (the engine owns all device
// memory), so their destructors free only what yalm allocated on the host.
#include "model.h"
#include "yalm_b200.h"

#include <cstdio>
#include <cstdlib>
#include <vector>

static yb_engine* g_b200 = nullptr;

static void b200_fail(const char* what, int rc) {
  char msg[512];
  yb_last_error(msg, sizeof(msg));
  std::fprintf(stderr, "b200 %s failed (%d): %s\n", what, rc, msg);
  std::abort();  // yalm's CLI aborts on device errors (CUDA_CHECK, src/infer.cu:14-22)
}

void yalm_b200_prepare(Model& m, int device) {
  const Config& c = *m.config;
  // yalm's DType order (src/codec.h:15-25): F16 = 1, F8E5M2 = 3
  yb_config cfg{c.dim, c.hidden_dim, c.head_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size,
                c.max_seq_len, c.rotary_dim, c.act == ActivationType::SILU ? 1 : 0, c.n_experts,
                static_cast<int>(c.weight_dtype), c.rope_theta, c.norm_eps, c.qkv_clip};
  const int L = c.n_layers;
  std::vector<const float*> att(L), ffn(L);
  std::vector<const uint16_t*> wq(L), wk(L), wv(L), wo(L), w1(L), w2(L), w3(L);
  for (int l = 0; l < L; ++l) {
    const Block& b = *m.blocks[l];
    att[l] = b.rms_att_weight();
    ffn[l] = b.rms_ffn_weight();
    wq[l] = b.wq<uint16_t>();
    wk[l] = b.wk<uint16_t>();
    wv[l] = b.wv<uint16_t>();
    wo[l] = b.wo<uint16_t>();
    w1[l] = b.w1<uint16_t>();
    w2[l] = b.w2<uint16_t>();
    w3[l] = b.w3<uint16_t>();
  }
  yb_weights w{static_cast<const uint16_t*>(m.token_embedding_table), m.rms_final_weight,
               static_cast<const uint16_t*>(m.wcls), att.data(), ffn.data(), wq.data(), wk.data(),
               wv.data(), wo.data(), w1.data(), w2.data(), w3.data()};
  if (int rc = yb_create(&cfg, &w, device, 0, 1, &g_b200)) b200_fail("yb_create", rc);
}

void yalm_b200_forward(Model& m, InferenceState& s, int token, int pos, InferenceMode mode) {
  (void)m;
  const int ybm = mode == InferenceMode::OUTPUT_LOGITS ? YB_MODE_OUTPUT_LOGITS : YB_MODE_HYDRATE_KV_CACHE;
  if (int rc = yb_forward(g_b200, token, pos, ybm, s.logits())) b200_fail("yb_forward", rc);
}
