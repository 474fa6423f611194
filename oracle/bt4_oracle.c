/*
 * bt4_oracle.c -- CPU restatement of the reference's BT4 forward pass.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * path (and the "port" CPU baseline of bench.py). It is never linked into the
 * product library; the product fails loudly when its CUDA library is missing.
 *
 * It restates, for the fixed attention-body topology of BT4-family networks,
 * the step-by-step fp32 interpretation that the reference's CPU backend runs
 * (src/nn/cpu/cpu_network.cpp RunBatch, :580-1491) over the execution plan of
 * src/nn/network_execution_plan.cpp:135-223. Every per-row loop keeps the
 * reference's accumulation order and float operations (no -ffast-math), so on
 * the same weights and inputs its outputs are bit-identical to the reference
 * binary built from the reference sources (checked by the golden fixtures).
 *
 * Positions are independent, so the batch is split over pthreads; each thread
 * runs one position at a time.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Activation kinds (src/nn/cpu/cpu_network.cpp:251-324). */
enum { ACT_NONE = 0, ACT_RELU, ACT_RELU2, ACT_TANH, ACT_SIGMOID, ACT_SWISH, ACT_MISH, ACT_SELU };

/* Global tensor slots; the order is mirrored by metalfish_b200/layout.py. */
enum {
  G_PREPROC_W, G_PREPROC_B, G_EMB_W, G_EMB_B, G_EMB_LN_G, G_EMB_LN_B, G_MULT_GATE, G_ADD_GATE,
  G_EFFN_W1, G_EFFN_B1, G_EFFN_W2, G_EFFN_B2, G_EFFN_LN_G, G_EFFN_LN_B, G_SMOLGEN_W,
  G_POL_W, G_POL_B, G_POL_WQ, G_POL_BQ, G_POL_WK, G_POL_BK, G_POL_PPO,
  G_VAL_W, G_VAL_B, G_VAL_W1, G_VAL_B1, G_VAL_W2, G_VAL_B2,
  G_MOV_W, G_MOV_B, G_MOV_W1, G_MOV_B1, G_MOV_W2, G_MOV_B2, G_COUNT
};
/* Per-encoder-layer tensor slots. */
enum {
  L_Q_W, L_Q_B, L_K_W, L_K_B, L_V_W, L_V_B, L_O_W, L_O_B,
  L_SG_COMPRESS, L_SG_W1, L_SG_B1, L_SG_LN1_G, L_SG_LN1_B, L_SG_W2, L_SG_B2, L_SG_LN2_G, L_SG_LN2_B,
  L_LN1_G, L_LN1_B, L_FFN_W1, L_FFN_B1, L_FFN_W2, L_FFN_B2, L_LN2_G, L_LN2_B, L_COUNT
};

typedef struct {
  int d, layers, heads, dff, emb_dff, pe;
  int sg_compress, sg_hidden, sg_gen;
  int dp, val_emb, val_hidden, mov_emb, mov_hidden;
  int act_default, act_smolgen, act_ffn;
} bt4o_config;

int bt4o_slot_counts(int *globals, int *per_layer) {
  *globals = G_COUNT;
  *per_layer = L_COUNT;
  return 0;
}

/* ActivationValue, src/nn/cpu/cpu_network.cpp:303-324. */
static float act(float v, int kind) {
  switch (kind) {
  case ACT_RELU: return v > 0.0f ? v : 0.0f;
  case ACT_RELU2: { const float r = v > 0.0f ? v : 0.0f; return r * r; }
  case ACT_TANH: return tanhf(v);
  case ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
  case ACT_SWISH: return v / (1.0f + expf(-v));
  case ACT_MISH: return v * tanhf(log1pf(expf(v)));
  case ACT_SELU: return 1.05070098f * (v > 0.0f ? v : 1.67326324f * (expf(v) - 1.0f));
  default: return v;
  }
}

static void act_n(float *x, size_t n, int kind) {
  if (kind == ACT_NONE) return;
  for (size_t i = 0; i < n; ++i) x[i] = act(x[i], kind);
}

/* DenseAffine, src/nn/cpu/cpu_network.cpp:382-403 (sum starts at the bias). */
static void dense(const float *in, int rows, int k, const float *w, const float *b, int n,
                  float *out) {
  for (int r = 0; r < rows; ++r) {
    const float *x = in + (size_t)r * k;
    float *y = out + (size_t)r * n;
    for (int o = 0; o < n; ++o) {
      const float *wr = w + (size_t)o * k;
      float s = b ? b[o] : 0.0f;
      for (int i = 0; i < k; ++i) s += x[i] * wr[i];
      y[o] = s;
    }
  }
}

/* ApplySoftmaxRows, src/nn/cpu/cpu_network.cpp:405-422. */
static void softmax_rows(float *v, int rows, int width) {
  for (int r = 0; r < rows; ++r) {
    float *x = v + (size_t)r * width;
    float m = -INFINITY;
    for (int c = 0; c < width; ++c) m = x[c] > m ? x[c] : m;
    float s = 0.0f;
    for (int c = 0; c < width; ++c) { x[c] = expf(x[c] - m); s += x[c]; }
    if (s == 0.0f) continue;
    const float inv = 1.0f / s;
    for (int c = 0; c < width; ++c) x[c] *= inv;
  }
}

/* ApplyLayerNorm, src/nn/cpu/cpu_network.cpp:424-460 (one-pass variance). */
static void layernorm(const float *in, const float *parent, float alpha, const float *g,
                      const float *b, float *out, int rows, int width, float eps) {
  for (int r = 0; r < rows; ++r) {
    const float *x = in + (size_t)r * width;
    const float *p = parent ? parent + (size_t)r * width : NULL;
    float *y = out + (size_t)r * width;
    float s = 0.0f, sq = 0.0f;
    for (int c = 0; c < width; ++c) {
      const float v = p ? p[c] + x[c] * alpha : x[c];
      s += v;
      sq += v * v;
    }
    const float mean = s / (float)width;
    float var = sq / (float)width - mean * mean;
    if (var < 0.0f) var = 0.0f;
    const float inv = 1.0f / sqrtf(var + eps);
    for (int c = 0; c < width; ++c) {
      const float v = p ? p[c] + x[c] * alpha : x[c];
      y[c] = (v - mean) * inv * g[c] + b[c];
    }
  }
}

/* Attention-policy gather table: raw index (64*64 + 8*24) -> policy index.
 * Generated from the move geometry of the 1858-entry policy encoding
 * (src/nn/policy_map.cpp kMoveStrings order; table src/nn/tables/
 * attention_policy_map.h:15): for every from-square in ascending order, every
 * to-square in ascending order that a queen or knight reaches; then the
 * underpromotions from the 7th rank, laid out as from_file*24 + to_file*3 +
 * piece, for |to_file - from_file| <= 1. */
int bt4o_build_policy_map(int16_t *table /* 4288 */) {
  int next = 0;
  for (int i = 0; i < 4288; ++i) table[i] = -1;
  for (int from = 0; from < 64; ++from) {
    const int fr = from / 8, ff = from % 8;
    for (int to = 0; to < 64; ++to) {
      if (to == from) continue;
      const int tr = to / 8, tf = to % 8;
      const int dr = tr - fr, df = tf - ff;
      const int adr = dr < 0 ? -dr : dr, adf = df < 0 ? -df : df;
      const int queen = dr == 0 || df == 0 || adr == adf;
      const int knight = (adr == 1 && adf == 2) || (adr == 2 && adf == 1);
      if (queen || knight) table[from * 64 + to] = (int16_t)next++;
    }
  }
  for (int ff = 0; ff < 8; ++ff)
    for (int tf = 0; tf < 8; ++tf)
      for (int piece = 0; piece < 3; ++piece) {
        const int df = tf - ff;
        if (df >= -1 && df <= 1) table[4096 + ff * 24 + tf * 3 + piece] = (int16_t)next++;
      }
  return next; /* 1858 */
}

/* Attention policy map, src/nn/cpu/cpu_network.cpp:892-1025: raw[q*64+k] =
 * (q.k) / sqrt(dq), the 8x24 promotion logits, then the 1858 gather. q and k
 * are [64, dq] for one position, ppo is ip4_pol_w [4, dq]. */
static int16_t g_gather[1858];
static pthread_once_t g_gather_once = PTHREAD_ONCE_INIT;
static void init_gather(void) {
  int16_t t[4288];
  bt4o_build_policy_map(t);
  for (int i = 0; i < 1858; ++i) g_gather[i] = -1;
  for (int r = 0; r < 4288; ++r)
    if (t[r] >= 0) g_gather[t[r]] = (int16_t)r;
}

void bt4o_policy_map(const float *q, const float *k, const float *ppo, int dq, float *out1858) {
  pthread_once(&g_gather_once, init_gather);
  const int16_t *gather = g_gather;
  float raw[4288];
  const float scale = 1.0f / sqrtf((float)dq);
  for (int qs = 0; qs < 64; ++qs)
    for (int ks = 0; ks < 64; ++ks) {
      float s = 0.0f;
      for (int c = 0; c < dq; ++c) s += q[qs * dq + c] * k[ks * dq + c];
      raw[qs * 64 + ks] = s * scale;
    }
  for (int promo = 0; promo < 192; ++promo) {
    const int prow = promo % 3;
    const int pks = 56 + (promo % 24) / 3;
    const int pair = promo % 64;
    const int qs = 48 + pair / 8;
    const int ks = 56 + pair % 8;
    float v = 0.0f;
    for (int c = 0; c < dq; ++c) {
      v += q[qs * dq + c] * k[ks * dq + c] * scale;
      v += k[pks * dq + c] * (ppo[prow * dq + c] + ppo[3 * dq + c]);
    }
    raw[4096 + promo] = v;
  }
  for (int p = 0; p < 1858; ++p) out1858[p] = gather[p] >= 0 ? raw[gather[p]] : 0.0f;
}

/* One attention block (src/nn/cpu/cpu_network.cpp:1037-1265) for one position:
 * x [64, d] -> out [64, d] (before the residual LN). */
static void attention(const bt4o_config *c, const float *const *L, const float *sgw,
                      const float *x, float *out, float *scratch) {
  const int d = c->d, H = c->heads, dh = d / H, T = 64;
  float *q = scratch, *k = q + T * d, *v = k + T * d;
  float *comp = v + T * d;                         /* [64, c] */
  float *h1 = comp + T * c->sg_compress;           /* [hidden] */
  float *n1 = h1 + c->sg_hidden;
  float *h2 = n1 + c->sg_hidden;                   /* [H*g] */
  float *n2 = h2 + H * c->sg_gen;
  float *bias = n2 + H * c->sg_gen;                /* [H, 64*64] */
  float *scores = bias + (size_t)H * T * T;        /* [H*64, 64] */
  float *ctx = scores + (size_t)H * T * T;         /* [64, d] */
  dense(x, T, d, L[L_Q_W], L[L_Q_B], d, q);
  dense(x, T, d, L[L_K_W], L[L_K_B], d, k);
  dense(x, T, d, L[L_V_W], L[L_V_B], d, v);
  /* smolgen (:1143-1172): dense + separate bias add, activation, LN eps 1e-3 */
  dense(x, T, d, L[L_SG_COMPRESS], NULL, c->sg_compress, comp);
  dense(comp, 1, T * c->sg_compress, L[L_SG_W1], NULL, c->sg_hidden, h1);
  for (int i = 0; i < c->sg_hidden; ++i) h1[i] += L[L_SG_B1][i];
  act_n(h1, (size_t)c->sg_hidden, c->act_smolgen);
  layernorm(h1, NULL, 1.0f, L[L_SG_LN1_G], L[L_SG_LN1_B], n1, 1, c->sg_hidden, 1e-3f);
  dense(n1, 1, c->sg_hidden, L[L_SG_W2], NULL, H * c->sg_gen, h2);
  for (int i = 0; i < H * c->sg_gen; ++i) h2[i] += L[L_SG_B2][i];
  act_n(h2, (size_t)H * c->sg_gen, c->act_smolgen);
  layernorm(h2, NULL, 1.0f, L[L_SG_LN2_G], L[L_SG_LN2_B], n2, 1, H * c->sg_gen, 1e-3f);
  dense(n2, H, c->sg_gen, sgw, NULL, T * T, bias);
  /* scores + bias, softmax, context (:1175-1254) */
  const float scale = 1.0f / sqrtf((float)dh);
  for (int h = 0; h < H; ++h)
    for (int qs = 0; qs < T; ++qs)
      for (int ks = 0; ks < T; ++ks) {
        float s = 0.0f;
        for (int e = 0; e < dh; ++e) s += q[qs * d + h * dh + e] * k[ks * d + h * dh + e];
        s *= scale;
        s += bias[(size_t)h * T * T + qs * T + ks];
        scores[((size_t)h * T + qs) * T + ks] = s;
      }
  softmax_rows(scores, H * T, T);
  for (int qs = 0; qs < T; ++qs)
    for (int h = 0; h < H; ++h) {
      const float *p = scores + ((size_t)h * T + qs) * T;
      for (int e = 0; e < dh; ++e) {
        float s = 0.0f;
        for (int ks = 0; ks < T; ++ks) s += p[ks] * v[ks * d + h * dh + e];
        ctx[qs * d + h * dh + e] = s;
      }
    }
  dense(ctx, T, d, L[L_O_W], L[L_O_B], d, out);
}

static size_t scratch_floats(const bt4o_config *c) {
  const size_t T = 64, d = (size_t)c->d, H = (size_t)c->heads;
  const size_t wide = (size_t)(c->dff > c->emb_dff ? c->dff : c->emb_dff);
  size_t attn = 3 * T * d + T * (size_t)c->sg_compress + 2 * (size_t)c->sg_hidden +
                2 * H * (size_t)c->sg_gen + 2 * H * T * T + T * d;
  size_t ffn = T * wide;
  size_t pol = 3 * T * (size_t)c->dp;
  size_t m = attn > ffn ? attn : ffn;
  return (m > pol ? m : pol) + 64;
}

/* Forward of one position, src/nn/cpu/cpu_network.cpp:580-1491 over the plan
 * of src/nn/network_execution_plan.cpp:155-223. */
static void forward_one(const bt4o_config *c, const float *const *G, const float *const *Ls,
                        const uint64_t *masks, const float *values, float *policy, float *wdl,
                        float *value, float *mlh, float *buf) {
  const int d = c->d, T = 64, P = 112;
  const size_t sc = scratch_floats(c);
  float *x = buf, *y = x + T * d, *t = y + T * d, *s = t + T * d;
  (void)sc;
  /* dynamic PE (:691-800): square-major 12-plane input, dense, concat */
  float pin[64 * 12];
  for (int sq = 0; sq < T; ++sq)
    for (int p = 0; p < 12; ++p)
      pin[sq * 12 + p] = ((masks[p] >> sq) & 1ULL) ? values[p] : 0.0f;
  float *pout = s;                                        /* [64*pe] */
  dense(pin, 1, T * 12, G[G_PREPROC_W], G[G_PREPROC_B], T * c->pe, pout);
  const int cw = P + c->pe;
  float *cat = pout + T * c->pe;                          /* [64, 112+pe] */
  for (int sq = 0; sq < T; ++sq) {
    for (int p = 0; p < P; ++p) cat[sq * cw + p] = ((masks[p] >> sq) & 1ULL) ? values[p] : 0.0f;
    for (int e = 0; e < c->pe; ++e) cat[sq * cw + P + e] = pout[sq * c->pe + e];
  }
  /* input embedding dense + default activation (:822-890, plan :1115-1116) */
  dense(cat, T, cw, G[G_EMB_W], G[G_EMB_B], d, t);
  act_n(t, (size_t)T * d, c->act_default);
  /* LN eps 1e-3 for PE_DENSE (plan :1175-1182) */
  layernorm(t, NULL, 1.0f, G[G_EMB_LN_G], G[G_EMB_LN_B], x, T, d, 1e-3f);
  /* gates, channel-major [d][64] (:1268-1316): multiply, then add */
  for (int r = 0; r < T; ++r)
    for (int col = 0; col < d; ++col) x[r * d + col] = x[r * d + col] * G[G_MULT_GATE][col * T + r];
  for (int r = 0; r < T; ++r)
    for (int col = 0; col < d; ++col) x[r * d + col] = x[r * d + col] + G[G_ADD_GATE][col * T + r];
  const float alpha = powf(2.0f * (float)c->layers, -0.25f); /* plan :1152-1162 */
  /* input embedding FFN + LN(x + alpha*ffn) eps 1e-3 (:1318-1397, :1423-1435) */
  {
    float *hid = s;
    dense(x, T, d, G[G_EFFN_W1], G[G_EFFN_B1], c->emb_dff, hid);
    act_n(hid, (size_t)T * c->emb_dff, c->act_ffn);
    dense(hid, T, c->emb_dff, G[G_EFFN_W2], G[G_EFFN_B2], d, t);
    layernorm(t, x, alpha, G[G_EFFN_LN_G], G[G_EFFN_LN_B], y, T, d, 1e-3f);
    float *sw = x; x = y; y = sw;
  }
  for (int l = 0; l < c->layers; ++l) {
    const float *const *L = Ls + (size_t)l * L_COUNT;
    attention(c, L, G[G_SMOLGEN_W], x, t, s);
    layernorm(t, x, alpha, L[L_LN1_G], L[L_LN1_B], y, T, d, 1e-3f); /* ln1 (:1436-1447) */
    float *hid = s;
    dense(y, T, d, L[L_FFN_W1], L[L_FFN_B1], c->dff, hid);
    act_n(hid, (size_t)T * c->dff, c->act_ffn);
    dense(hid, T, c->dff, L[L_FFN_W2], L[L_FFN_B2], d, t);
    layernorm(t, y, alpha, L[L_LN2_G], L[L_LN2_B], x, T, d, 1e-3f); /* ln2 */
  }
  /* attention policy head (plan :192-211; activations :1083-1096) */
  {
    const int dp = c->dp;
    float *e = s, *q = e + T * dp, *k = q + T * dp;
    dense(x, T, d, G[G_POL_W], G[G_POL_B], dp, e);
    act_n(e, (size_t)T * dp, c->act_default);
    dense(e, T, dp, G[G_POL_WQ], G[G_POL_BQ], dp, q);
    dense(e, T, dp, G[G_POL_WK], G[G_POL_BK], dp, k);
    bt4o_policy_map(q, k, G[G_POL_PPO], dp, policy);
  }
  /* value head (plan :213-223, :1098-1106): per square, flatten, softmax WDL */
  {
    float *ve = s, *v1 = ve + T * c->val_emb;
    dense(x, T, d, G[G_VAL_W], G[G_VAL_B], c->val_emb, ve);
    act_n(ve, (size_t)T * c->val_emb, c->act_default);
    dense(ve, 1, T * c->val_emb, G[G_VAL_W1], G[G_VAL_B1], c->val_hidden, v1);
    act_n(v1, (size_t)c->val_hidden, c->act_default);
    dense(v1, 1, c->val_hidden, G[G_VAL_W2], G[G_VAL_B2], 3, wdl);
    softmax_rows(wdl, 1, 3);
    *value = wdl[0] - wdl[2]; /* src/nn/network_output_decoder.cpp:60-66 */
  }
  /* moves-left head (plan :184-190, :1108-1111) */
  {
    float *me = s, *m1 = me + T * c->mov_emb;
    dense(x, T, d, G[G_MOV_W], G[G_MOV_B], c->mov_emb, me);
    act_n(me, (size_t)T * c->mov_emb, c->act_default);
    dense(me, 1, T * c->mov_emb, G[G_MOV_W1], G[G_MOV_B1], c->mov_hidden, m1);
    act_n(m1, (size_t)c->mov_hidden, c->act_default);
    dense(m1, 1, c->mov_hidden, G[G_MOV_W2], G[G_MOV_B2], 1, mlh);
    act_n(mlh, 1, ACT_RELU);
  }
}

typedef struct {
  const bt4o_config *c;
  const float *const *G, *const *L;
  const uint64_t *masks;
  const float *values;
  float *policy, *wdl, *value, *mlh;
  int lo, hi, status;
} job_t;

static void *worker(void *arg) {
  job_t *j = (job_t *)arg;
  const bt4o_config *c = j->c;
  const size_t n = 3 * 64 * (size_t)c->d + scratch_floats(c) + 64 * (size_t)(112 + c->pe) +
                   64 * (size_t)c->pe + 256;
  float *buf = (float *)malloc(n * sizeof(float));
  if (!buf) { j->status = -1; return NULL; }
  for (int b = j->lo; b < j->hi; ++b)
    forward_one(c, j->G, j->L, j->masks + (size_t)b * 112, j->values + (size_t)b * 112,
                j->policy + (size_t)b * 1858, j->wdl + (size_t)b * 3, j->value + b, j->mlh + b,
                buf);
  free(buf);
  return NULL;
}

/* Batched forward. G: G_COUNT tensor pointers; L: layers * L_COUNT pointers. */
int bt4o_forward(const bt4o_config *c, const float *const *G, const float *const *L,
                 const uint64_t *masks, const float *values, int batch, float *policy, float *wdl,
                 float *value, float *mlh, int threads) {
  if (batch <= 0) return 0;
  if (threads < 1) threads = 1;
  if (threads > batch) threads = batch;
  pthread_t tid[256];
  job_t jobs[256];
  if (threads > 256) threads = 256;
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (job_t){c, G, L, masks, values, policy, wdl, value, mlh,
                      (int)((int64_t)batch * t / threads), (int)((int64_t)batch * (t + 1) / threads), 0};
    pthread_create(&tid[t], NULL, worker, &jobs[t]);
  }
  int status = 0;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tid[t], NULL);
    if (jobs[t].status) status = jobs[t].status;
  }
  return status;
}

/* ---------------------------------------------------------------- priors
 * The step after the forward on the MCTS leaf path: the evaluator gathers
 * the raw policy logit of each legal move (src/mcts/evaluator.cpp:182-226;
 * an index outside [0, 1858) gives logit 0) and ApplyNNPolicyToNode turns
 * them into edge priors (src/mcts/search.cpp:127-197, the non-Apple branch):
 * n = min(moves, 256) (kMaxEdges, search.cpp:49), max over the n logits,
 * e_i = FastExp((l_i - max) * (1/temp)), sum in move order, uniform 1/n when
 * the sum is not positive, else e_i * (1/sum).
 *
 * FastExp (src/mcts/core.h:38-44) is Schraudolph's exponential (N. N.
 * Schraudolph, "A fast, compact approximation of the exponential function",
 * Neural Computation 11(4), 1999): clamp to [-88, 88], then the float whose
 * bits are the integer part of x * 2^23/ln 2 (12102203) plus the exponent
 * bias 127 << 23. */
float bt4o_fast_exp(float x) {
  x = x < 88.0f ? x : 88.0f;    /* std::min(88, x): a NaN x gives 88 */
  x = -88.0f < x ? x : -88.0f;  /* std::max(-88, x) */
  const int32_t i = (int32_t)(x * 12102203.0f) + 1065353216;
  float r;
  memcpy(&r, &i, sizeof r);
  return r;
}

/* policy [batch, 1858]; offsets [batch + 1] (CSR over index); priors has
 * offsets[batch] entries; moves past the 256th of a position get 0. */
void bt4o_priors(const float *policy, int batch, const int32_t *offsets, const int16_t *index,
                 float temp, float *priors) {
  const float inv_temp = 1.0f / temp;
  for (int b = 0; b < batch; ++b) {
    const int32_t lo = offsets[b];
    const int moves = offsets[b + 1] - lo;
    const int n = moves < 256 ? moves : 256;
    for (int i = n; i < moves; ++i) priors[lo + i] = 0.0f;
    if (n == 0) continue;
    float logit[256];
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) {
      const int idx = index[lo + i];
      logit[i] = (idx >= 0 && idx < 1858) ? policy[(size_t)b * 1858 + idx] : 0.0f;
      if (logit[i] > mx) mx = logit[i];
    }
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
      priors[lo + i] = bt4o_fast_exp((logit[i] - mx) * inv_temp);
      sum += priors[lo + i];
    }
    if (sum <= 0.0f) {
      const float u = 1.0f / (float)n;
      for (int i = 0; i < n; ++i) priors[lo + i] = u;
      continue;
    }
    const float inv_sum = 1.0f / sum;
    for (int i = 0; i < n; ++i) priors[lo + i] *= inv_sum;
  }
}

/* ---------------------------------------------------------------- encoder
 * NN::EncodePositionForNN (src/nn/encoder.cpp:249-466) for FillEmptyHistory
 * FEN_ONLY and 8 history planes, followed by PackInputPlaneRaw
 * (src/nn/input_plane_packing.h:30-61). The history is one record per
 * position, oldest first; the last record is the position evaluated. This
 * restatement builds the float planes exactly as the reference does and then
 * packs them, so it checks the GPU encoder (which works on bitboards) from a
 * different representation. One deliberate difference: a synthesised
 * history (before the first record) is cut after 8 entries, where the
 * reference would loop forever on a V2 format whose oldest record is not
 * the start position, has a nonzero rule50 and no repetition. */
typedef struct {
  uint64_t pieces[2][6]; /* [white, black][pawn, knight, bishop, rook, queen, king] */
  int32_t rule50, game_ply;
  int8_t ep_square;      /* -1: none */
  uint8_t castling;      /* 1 white O-O, 2 white O-O-O, 4 black O-O, 8 black O-O-O */
  uint8_t black_to_move, repetition;
  uint32_t reserved;
} bt4o_board;

int bt4o_board_size(void) { return (int)sizeof(bt4o_board); }

enum { T_FLIP = 1, T_MIRROR = 2, T_TRANSPOSE = 4 };
enum { C_WOO = 1, C_WOOO = 2, C_BOO = 4, C_BOOO = 8 };

/* encoder.cpp:46-51 */
static uint64_t rev_bits_in_bytes(uint64_t v) {
  v = ((v >> 1) & 0x5555555555555555ull) | ((v & 0x5555555555555555ull) << 1);
  v = ((v >> 2) & 0x3333333333333333ull) | ((v & 0x3333333333333333ull) << 2);
  v = ((v >> 4) & 0x0F0F0F0F0F0F0F0Full) | ((v & 0x0F0F0F0F0F0F0F0Full) << 4);
  return v;
}
/* encoder.cpp:53-58: byte order reversed (ranks mirrored) */
static uint64_t rev_bytes(uint64_t v) {
  v = (v & 0x00000000FFFFFFFFull) << 32 | (v & 0xFFFFFFFF00000000ull) >> 32;
  v = (v & 0x0000FFFF0000FFFFull) << 16 | (v & 0xFFFF0000FFFF0000ull) >> 16;
  v = (v & 0x00FF00FF00FF00FFull) << 8 | (v & 0xFF00FF00FF00FF00ull) >> 8;
  return v;
}
/* encoder.cpp:60-68: the 8x8 bit matrix transposed (files <-> ranks) */
static uint64_t transpose_bits(uint64_t v) {
  v = (v & 0xAA00AA00AA00AA00ull) >> 9 | (v & 0x0055005500550055ull) << 9 | (v & 0x55AA55AA55AA55AAull);
  v = (v & 0xCCCC0000CCCC0000ull) >> 18 | (v & 0x0000333300003333ull) << 18 | (v & 0x3333CCCC3333CCCCull);
  v = (v & 0xF0F0F0F000000000ull) >> 36 | (v & 0x000000000F0F0F0Full) << 36 | (v & 0x0F0F0F0FF0F0F0F0ull);
  return v;
}
/* encoder.cpp:70-86 */
static uint64_t apply_transform(uint64_t b, int t) {
  if (b == 0 || b == ~0ull) return b;
  if (t & T_FLIP) b = rev_bits_in_bytes(b);
  if (t & T_MIRROR) b = rev_bytes(b);
  if (t & T_TRANSPOSE) b = transpose_bits(b);
  return b;
}
/* encoder.cpp:88-102 */
static int compare_transposing(uint64_t board, int t) {
  uint64_t v = board;
  if (t & T_FLIP) v = rev_bits_in_bytes(v);
  if (t & T_MIRROR) v = rev_bytes(v);
  const uint64_t alt = transpose_bits(v);
  return v < alt ? -1 : (v > alt ? 1 : 0);
}
static uint64_t kind(const bt4o_board *p, int k) { return p->pieces[0][k] | p->pieces[1][k]; }
static uint64_t side(const bt4o_board *p, int c) {
  uint64_t b = 0;
  for (int k = 0; k < 6; ++k) b |= p->pieces[c][k];
  return b;
}
/* encoder.cpp:104-170 */
static int choose_transform(const bt4o_board *p, int us) {
  if (p->castling) return 0;
  uint64_t king = p->pieces[us][5];
  int t = 0;
  if (king & 0x0F0F0F0F0F0F0F0Full) {
    t |= T_FLIP;
    king = rev_bits_in_bytes(king);
  }
  if (kind(p, 0)) return t;
  if (king & 0xFFFFFFFF00000000ull) {
    t |= T_MIRROR;
    king = rev_bytes(king);
  }
  if (king & 0xE0C08000ull) return t | T_TRANSPOSE;
  if (king & 0x10204080ull) {
    /* tie-breaks in the reference's order: all pieces, ours, kings, queens,
       rooks, knights, bishops */
    const uint64_t order[7] = {side(p, 0) | side(p, 1), side(p, us), kind(p, 5), kind(p, 4),
                               kind(p, 3), kind(p, 1), kind(p, 2)};
    for (int i = 0; i < 7; ++i) {
      const int o = compare_transposing(order[i], t);
      if (o == -1) return t;
      if (o == 1) return t | T_TRANSPOSE;
    }
  }
  return t;
}
/* encoder.cpp:214-238 (IsStartPosition) */
static int is_start(const bt4o_board *p) {
  static const uint64_t start[2][6] = {
      {0x000000000000FF00ull, 0x42ull, 0x24ull, 0x81ull, 0x08ull, 0x10ull},
      {0x00FF000000000000ull, 0x4200000000000000ull, 0x2400000000000000ull,
       0x8100000000000000ull, 0x0800000000000000ull, 0x1000000000000000ull}};
  if (p->black_to_move || p->game_ply != 0 || p->rule50 != 0 || p->ep_square >= 0 ||
      p->castling != 15)
    return 0;
  for (int c = 0; c < 2; ++c)
    for (int k = 0; k < 6; ++k)
      if (p->pieces[c][k] != start[c][k]) return 0;
  return 1;
}
/* encoder.cpp:338-360: castling rights, our side first */
static int castle_mask_for(const bt4o_board *p, int us) {
  const int c = p->castling;
  if (!us) return ((c & C_WOO) ? 1 : 0) | ((c & C_WOOO) ? 2 : 0) | ((c & C_BOO) ? 4 : 0) | ((c & C_BOOO) ? 8 : 0);
  return ((c & C_BOO) ? 1 : 0) | ((c & C_BOOO) ? 2 : 0) | ((c & C_WOO) ? 4 : 0) | ((c & C_WOOO) ? 8 : 0);
}

static void set_plane(float *pl, float v) {
  for (int s = 0; s < 64; ++s) pl[s] = v;
}
static void set_bits(float *pl, uint64_t b) {
  for (int s = 0; s < 64; ++s)
    if ((b >> s) & 1) pl[s] = 1.0f;
}
static void fill_from(float *pl, uint64_t b) {
  set_plane(pl, 0.0f);
  set_bits(pl, b);
}

static void encode_one(const bt4o_board *h, int n, int fmt, float (*r)[64], int *transform_out) {
  memset(r, 0, sizeof(float) * 112 * 64);
  *transform_out = 0;
  if (n <= 0) return;
  const bt4o_board *cur = &h[n - 1];
  const int us = cur->black_to_move, them = !us;
  const int canonical = fmt == 3 || fmt == 4 || fmt == 5 || fmt == 132 || fmt == 133;
  const int v2 = fmt == 5 || fmt == 133;
  const int hecto = fmt == 4 || fmt == 132 || fmt == 5 || fmt == 133;
  const int arma = fmt == 132 || fmt == 133;
  const int transform = canonical ? choose_transform(cur, us) : 0;
  const int A = 104;
  /* auxiliary planes, encoder.cpp:279-336 */
  if (fmt == 1) {
    const int oq = us ? C_BOOO : C_WOOO, ok = us ? C_BOO : C_WOO;
    const int tq = us ? C_WOOO : C_BOOO, tk = us ? C_WOO : C_BOO;
    set_plane(r[A + 0], (cur->castling & oq) ? 1.0f : 0.0f);
    set_plane(r[A + 1], (cur->castling & ok) ? 1.0f : 0.0f);
    set_plane(r[A + 2], (cur->castling & tq) ? 1.0f : 0.0f);
    set_plane(r[A + 3], (cur->castling & tk) ? 1.0f : 0.0f);
  } else {
    const int c = cur->castling;
    if (!us) {
      if (c & C_WOOO) r[A + 0][0] = 1.0f;
      if (c & C_WOO) r[A + 1][7] = 1.0f;
      if (c & C_BOOO) r[A + 0][56] = 1.0f;
      if (c & C_BOO) r[A + 1][63] = 1.0f;
    } else {
      if (c & C_BOOO) r[A + 0][0] = 1.0f;
      if (c & C_BOO) r[A + 1][7] = 1.0f;
      if (c & C_WOOO) r[A + 0][56] = 1.0f;
      if (c & C_WOO) r[A + 1][63] = 1.0f;
    }
  }
  if (canonical) {
    if (cur->ep_square >= 0) r[A + 4][cur->ep_square] = 1.0f;
  } else {
    set_plane(r[A + 4], us ? 1.0f : 0.0f);
  }
  set_plane(r[A + 5], hecto ? (float)cur->rule50 / 100.0f : (float)cur->rule50);
  set_plane(r[A + 6], (arma && us) ? 1.0f : 0.0f);
  set_plane(r[A + 7], 1.0f);
  /* history, encoder.cpp:362-437 */
  const int root_mask = castle_mask_for(cur, us);
  for (int i = 0, hi = n - 1; i < 8; ++i, --hi) {
    if (hi < -8) break; /* see the header comment */
    const bt4o_board *p = &h[hi >= 0 ? hi : 0];
    if (hi < 0 && is_start(p)) break;
    if (canonical && hi < n - 1) {
      if (castle_mask_for(p, us) != root_mask) break;
      if (p->ep_square >= 0) break;
    }
    const int rep = p->repetition != 0;
    if (v2 && i > 0 && !rep) {
      if (p->rule50 == 0) break;
      --i;
      continue;
    }
    const int base = i * 13;
    uint64_t our[6], their[6];
    for (int k = 0; k < 6; ++k) {
      our[k] = p->pieces[us][k];
      their[k] = p->pieces[them][k];
      if (us) {
        our[k] = rev_bytes(our[k]);
        their[k] = rev_bytes(their[k]);
      }
    }
    for (int k = 0; k < 6; ++k) set_bits(r[base + k], our[k]);
    for (int k = 0; k < 6; ++k) set_bits(r[base + 6 + k], their[k]);
    set_plane(r[base + 12], rep ? 1.0f : 0.0f);
    if (hi < 0 && p->ep_square >= 0) {
      const int e = p->ep_square;
      if (e < 8)
        fill_from(r[base + 0], our[0] + ((0x0000000000000100ull - 0x0000000001000000ull) << e));
      else if (e >= 56)
        fill_from(r[base + 6], their[0] + ((0x0001000000000000ull - 0x0000000100000000ull) << (e - 56)));
    }
    if (canonical && p->rule50 == 0) break;
  }
  /* canonicalisation, encoder.cpp:439-455 */
  if (transform) {
    for (int i = 0; i <= A + 4; ++i) {
      uint64_t b = 0;
      for (int s = 0; s < 64; ++s)
        if (r[i][s] > 0.5f) b |= 1ull << s;
      if (b == 0 || b == ~0ull) continue;
      fill_from(r[i], apply_transform(b, transform));
    }
  }
  *transform_out = transform;
}

/* PackInputPlaneRaw (input_plane_packing.h:30-61) */
static void pack_plane(const float *pl, int p, uint64_t *mask, float *value) {
  const int uniform = (p < 104 && p % 13 == 12) || p == 106 || p == 107 || p >= 109;
  if (uniform) {
    *value = pl[0];
    *mask = *value != 0.0f ? ~0ull : 0ull;
    return;
  }
  *mask = 0;
  *value = 0.0f;
  for (int s = 0; s < 64; ++s)
    if (pl[s] != 0.0f) {
      if (*mask == 0) *value = pl[s];
      *mask |= 1ull << s;
    }
}

int bt4o_encode(const bt4o_board *boards, const int32_t *offsets, int batch, int fmt,
                uint64_t *masks, float *values, int32_t *transforms) {
  float (*r)[64] = (float (*)[64])malloc(sizeof(float) * 112 * 64);
  if (!r) return 1;
  for (int b = 0; b < batch; ++b) {
    int t = 0;
    encode_one(boards + (offsets[b] - offsets[0]), offsets[b + 1] - offsets[b], fmt, r, &t);
    for (int p = 0; p < 112; ++p)
      pack_plane(r[p], p, &masks[(size_t)b * 112 + p], &values[(size_t)b * 112 + p]);
    if (transforms) transforms[b] = t;
  }
  free(r);
  return 0;
}
