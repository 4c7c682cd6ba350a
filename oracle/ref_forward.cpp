// ref_forward.cpp — oracle (TEST INFRASTRUCTURE ONLY): a C++ restatement of the
// reference decode path with the reference's loop order, used to cross-check
// ref_forward.py and as the timed CPU baseline. Not part of the product: only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
//
// Follows, loop for loop:
//   MATMUL    kernels.js:26-44   one output per (t, j); k ascends in steps of 4,
//                                 acc = acc + x*w as separate fp32 mul and add
//   RMSNORM   kernels.js:46-63   ss ascends over i; scale = 1/sqrt(ss/d + 1e-6)
//   ROPE      kernels.js:66-83   freq = exp2(-2*half/hd*log2(theta)); ang = f32(pos)*freq
//   ATTENTION kernels.js:86-132  pass 1 online max/sum from maxs = -3e30, pass 2
//                                 w = exp(s - maxs)/sume, acc[e] += V*w
//   SILUMUL   kernels.js:134-145 a / (1 + exp(-a)) * b
//   ADDBIAS / ADD kernels.js:148-171
//   Stage.forward pipeline.js:48-78, appendKv :80-87, sampleLast :141-174,
//   generate :255-281.
// Parallelism (std::thread, static partition) only splits independent outputs,
// so results do not depend on the thread count. Built with -ffp-contract=off so no mul+add pair is
// fused. Transcendentals: double-precision libm rounded to float.
// Parity status: unpinned (the reference cannot run on this machine).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace {

int g_threads = 1;

// Run f(i) for i in [0, n) on g_threads threads, contiguous static blocks.
template <typename F>
void par_for(long long n, F f) {
  const int nt = (int)std::max(1ll, std::min<long long>(g_threads, n / 64 + 1));
  if (nt <= 1) {
    for (long long i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> th;
  th.reserve(nt);
  for (int w = 0; w < nt; ++w) {
    const long long lo = n * w / nt, hi = n * (w + 1) / nt;
    th.emplace_back([lo, hi, &f] {
      for (long long i = lo; i < hi; ++i) f(i);
    });
  }
  for (auto& t : th) t.join();
}

inline float bf(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

inline float hash_normal(uint64_t seed, uint64_t i) {
  const uint64_t r = mix64(mix64(seed) ^ i);
  const float u1 = ((float)(r >> 40) + 1.0f) * 5.9604644775390625e-8f;
  const float u2 = (float)(r & 0xffffffull) * 5.9604644775390625e-8f;
  return (float)(std::sqrt(-2.0 * std::log((double)u1)) * std::cos(2.0 * M_PI * (double)u2));
}

}  // namespace

extern "C" {

int ref_num_threads(void) { return g_threads; }

void ref_set_threads(int n) {
  if (n > 0) g_threads = n;
}

// ---- shaders -----------------------------------------------------------------------
void ref_matmul(const float* x, const uint16_t* w, float* out, int n, int din, int dout) {
  for (int t = 0; t < n; ++t) {
    const float* xr = x + (size_t)t * din;
    par_for(dout, [&](long long jj) {
      const int j = (int)jj;
      const uint16_t* wr = w + (size_t)j * din;
      float acc = 0.0f;
      int k = 0;
      for (; k + 3 < din; k += 4) {
        acc = acc + xr[k] * bf(wr[k]);
        acc = acc + xr[k + 1] * bf(wr[k + 1]);
        acc = acc + xr[k + 2] * bf(wr[k + 2]);
        acc = acc + xr[k + 3] * bf(wr[k + 3]);
      }
      for (; k < din; ++k) acc = acc + xr[k] * bf(wr[k]);
      out[(size_t)t * dout + j] = acc;
    });
  }
}

void ref_rmsnorm(const float* x, const uint16_t* g, float* out, int n, int d, float eps) {
  for (int t = 0; t < n; ++t) {
    const float* xr = x + (size_t)t * d;
    float ss = 0.0f;
    for (int i = 0; i < d; ++i) ss = ss + xr[i] * xr[i];
    const float scale = 1.0f / std::sqrt(ss / (float)d + eps);
    for (int i = 0; i < d; ++i) out[(size_t)t * d + i] = xr[i] * scale * bf(g[i]);
  }
}

void ref_rope_freqs(int hd, float theta, float* freq) {
  const float l2t = (float)std::log2((double)theta);
  for (int h = 0; h < hd / 2; ++h) {
    const float e = (-2.0f * (float)h) / (float)hd * l2t;
    freq[h] = (float)std::exp2((double)e);
  }
}

void ref_rope(float* x, int n, int heads, int hd, int pos0, const float* freq) {
  const int half = hd / 2;
  for (int t = 0; t < n; ++t) {
    const float pos = (float)(pos0 + t);
    for (int h = 0; h < heads; ++h) {
      float* row = x + (size_t)t * heads * hd + (size_t)h * hd;
      for (int i = 0; i < half; ++i) {
        const float ang = pos * freq[i];
        const float c = (float)std::cos((double)ang), s = (float)std::sin((double)ang);
        const float x1 = row[i], x2 = row[i + half];
        row[i] = x1 * c - x2 * s;
        row[i + half] = x1 * s + x2 * c;
      }
    }
  }
}

// caches: [max_pos][kvh*hd] fp32
void ref_attention(const float* q, const float* kc, const float* vc, float* out, int T0, int n, int nq, int kvh,
                   int hd) {
  const float scale = (float)(1.0 / std::sqrt((double)hd));
  const int grp = nq / kvh;
  par_for((long long)n * nq, [&](long long th) {
    {
      const int t = (int)(th / nq), h = (int)(th % nq);
      const int g = h / grp;
      const int tend = T0 + t + 1;
      const float* qr = q + (size_t)t * nq * hd + (size_t)h * hd;
      float maxs = -3.0e30f, sume = 0.0f;
      for (int p = 0; p < tend; ++p) {
        const float* kr = kc + (size_t)p * kvh * hd + (size_t)g * hd;
        float s = 0.0f;
        for (int e = 0; e < hd; ++e) s = s + qr[e] * kr[e];
        s = s * scale;
        if (s > maxs) {
          if (sume > 0.0f) sume = sume * (float)std::exp((double)(maxs - s));
          maxs = s;
        }
        sume = sume + (float)std::exp((double)(s - maxs));
      }
      std::vector<float> acc(hd, 0.0f);
      for (int p = 0; p < tend; ++p) {
        const float* kr = kc + (size_t)p * kvh * hd + (size_t)g * hd;
        float s = 0.0f;
        for (int e = 0; e < hd; ++e) s = s + qr[e] * kr[e];
        s = s * scale;
        const float w = (float)std::exp((double)(s - maxs)) / sume;
        const float* vr = vc + (size_t)p * kvh * hd + (size_t)g * hd;
        for (int e = 0; e < hd; ++e) acc[e] = acc[e] + vr[e] * w;
      }
      float* o = out + (size_t)t * nq * hd + (size_t)h * hd;
      for (int e = 0; e < hd; ++e) o[e] = acc[e];
    }
  });
}

void ref_silu_mul(const float* a, const float* b, float* out, int total) {
  par_for(total, [&](long long i) {
    const float v = a[i];
    out[i] = v / (1.0f + (float)std::exp((double)-v)) * b[i];
  });
}

void ref_add(const float* a, const float* b, float* out, int total) {
  for (int i = 0; i < total; ++i) out[i] = a[i] + b[i];
}

void ref_add_bias(const float* a, const uint16_t* bias, float* out, int n, int dout) {
  for (int i = 0; i < n * dout; ++i) out[i] = a[i] + bf(bias[i % dout]);
}

// Fill n bf16 values from the counter hash used by the synthetic KV/weights of the bench.
void ref_fill_normal_bf16(uint16_t* p, size_t n, uint64_t seed, float std) {
  par_for((long long)n, [&](long long i) { p[i] = to_bf16(hash_normal(seed, (uint64_t)i) * std); });
}

// ---- model -------------------------------------------------------------------------------
struct RefModel {
  int D, NQ, KVH, HD, I, V, L0, L1, max_pos, kv_bf16;
  float eps, theta;
  std::vector<const uint16_t*> w;  // 12 per layer in tensorsForLayers order
  const uint16_t *embed, *norm, *lm_head;
  std::vector<std::vector<float>> kk, vv;  // per local layer [max_pos][KVH*HD]
  std::vector<float> freq;
  int T0;
};

// dims: D, NQ, KVH, HD, I, V, start, end, max_pos, kv_bf16
// layer_w: (end-start)*12 pointers (biases may be null); head pointers may be null.
void* ref_model_create(const int* dims, float eps, float theta, const uint16_t* const* layer_w, const uint16_t* embed,
                       const uint16_t* norm, const uint16_t* lm_head) {
  auto* m = new RefModel();
  m->D = dims[0];
  m->NQ = dims[1];
  m->KVH = dims[2];
  m->HD = dims[3];
  m->I = dims[4];
  m->V = dims[5];
  m->L0 = dims[6];
  m->L1 = dims[7];
  m->max_pos = dims[8];
  m->kv_bf16 = dims[9];
  m->eps = eps;
  m->theta = theta;
  const int nl = m->L1 - m->L0;
  m->w.assign(layer_w, layer_w + (size_t)nl * 12);
  m->embed = embed;
  m->norm = norm;
  m->lm_head = lm_head;
  m->kk.assign(nl, std::vector<float>((size_t)m->max_pos * m->KVH * m->HD, 0.0f));
  m->vv.assign(nl, std::vector<float>((size_t)m->max_pos * m->KVH * m->HD, 0.0f));
  m->freq.resize(m->HD / 2);
  ref_rope_freqs(m->HD, theta, m->freq.data());
  m->T0 = 0;
  return m;
}

void ref_model_destroy(void* h) { delete (RefModel*)h; }
int ref_model_t0(void* h) { return ((RefModel*)h)->T0; }
void ref_model_set_t0(void* h, int t0) { ((RefModel*)h)->T0 = t0; }

// Synthetic prefilled KV: n slots of N(0,1) (bf16-rounded when the cache is bf16).
void ref_model_fill_kv(void* h, int n, uint64_t seed) {
  auto* m = (RefModel*)h;
  const size_t row = (size_t)m->KVH * m->HD;
  for (size_t l = 0; l < m->kk.size(); ++l) {
    par_for((long long)n * (long long)row, [&](long long i) {
      float a = hash_normal(seed + 2 * l, (uint64_t)i), b = hash_normal(seed + 2 * l + 1, (uint64_t)i);
      if (m->kv_bf16) {
        a = bf(to_bf16(a));
        b = bf(to_bf16(b));
      }
      m->kk[l][i] = a;
      m->vv[l][i] = b;
    });
  }
  m->T0 = n;
}

// Load KV rows into slots [slot0, slot0 + n) of local layer `layer` (which: 0 = K,
// 1 = V) from src [n][KVH*HD] fp32, bf16-rounded when the cache is bf16. Lets a
// check start from the exact cache contents another implementation holds.
int ref_model_set_kv(void* h, int layer, int which, int slot0, int n, const float* src) {
  auto* m = (RefModel*)h;
  if (layer < 0 || layer >= (int)m->kk.size() || slot0 < 0 || n < 0 || slot0 + n > m->max_pos) return -1;
  const size_t row = (size_t)m->KVH * m->HD;
  std::vector<float>& dst = which ? m->vv[layer] : m->kk[layer];
  for (size_t i = 0; i < (size_t)n * row; ++i) {
    float a = src[i];
    if (m->kv_bf16) a = bf(to_bf16(a));
    dst[(size_t)slot0 * row + i] = a;
  }
  return 0;
}

// Stage.forward (pipeline.js:48-78): h [n][D] in place. Returns 0, or -1 on KV overflow.
int ref_stage_forward(void* hm, float* h, int n, int pos_start) {
  auto* m = (RefModel*)hm;
  const int D = m->D, QD = m->NQ * m->HD, KD = m->KVH * m->HD, I = m->I;
  if (m->T0 + n > m->max_pos) return -1;
  std::vector<float> x((size_t)n * D), q((size_t)n * QD), k((size_t)n * KD), v((size_t)n * KD), att((size_t)n * QD),
      o((size_t)n * D), g((size_t)n * I), u((size_t)n * I), mm((size_t)n * I), d((size_t)n * D);
  for (int L = 0; L < m->L1 - m->L0; ++L) {
    const uint16_t* const* W = &m->w[(size_t)L * 12];
    ref_rmsnorm(h, W[0], x.data(), n, D, m->eps);
    ref_matmul(x.data(), W[2], q.data(), n, D, QD);
    ref_matmul(x.data(), W[3], k.data(), n, D, KD);
    ref_matmul(x.data(), W[4], v.data(), n, D, KD);
    if (W[6]) ref_add_bias(q.data(), W[6], q.data(), n, QD);
    if (W[7]) ref_add_bias(k.data(), W[7], k.data(), n, KD);
    if (W[8]) ref_add_bias(v.data(), W[8], v.data(), n, KD);
    ref_rope(q.data(), n, m->NQ, m->HD, pos_start, m->freq.data());
    ref_rope(k.data(), n, m->KVH, m->HD, pos_start, m->freq.data());
    for (size_t i = 0; i < (size_t)n * KD; ++i) {  // appendKv (pipeline.js:80-87)
      float a = k[i], b = v[i];
      if (m->kv_bf16) {
        a = bf(to_bf16(a));
        b = bf(to_bf16(b));
      }
      m->kk[L][(size_t)m->T0 * KD + i] = a;
      m->vv[L][(size_t)m->T0 * KD + i] = b;
    }
    ref_attention(q.data(), m->kk[L].data(), m->vv[L].data(), att.data(), m->T0, n, m->NQ, m->KVH, m->HD);
    ref_matmul(att.data(), W[5], o.data(), n, QD, D);
    ref_add(h, o.data(), h, n * D);
    ref_rmsnorm(h, W[1], x.data(), n, D, m->eps);
    ref_matmul(x.data(), W[9], g.data(), n, D, I);
    ref_matmul(x.data(), W[10], u.data(), n, D, I);
    ref_silu_mul(g.data(), u.data(), mm.data(), n * I);
    ref_matmul(mm.data(), W[11], d.data(), n, I, D);
    ref_add(h, d.data(), h, n * D);
  }
  m->T0 += n;
  return 0;
}

// sampleLast (pipeline.js:141-174): norm, LM head in 8192-row chunks, strict '>' scan.
int ref_sample_last(void* hm, const float* hrow, float* logits_out) {
  auto* m = (RefModel*)hm;
  const int D = m->D;
  std::vector<float> nrm(D), lg(m->V);
  ref_rmsnorm(hrow, m->norm, nrm.data(), 1, D, m->eps);
  const uint16_t* E = m->lm_head ? m->lm_head : m->embed;
  for (int r0 = 0; r0 < m->V; r0 += 8192) {
    const int rows = std::min(8192, m->V - r0);
    ref_matmul(nrm.data(), E + (size_t)r0 * D, lg.data() + r0, 1, D, rows);
  }
  int best = 0;
  float bestv = -INFINITY;
  for (int i = 0; i < m->V; ++i)
    if (lg[i] > bestv) {
      bestv = lg[i];
      best = i;
    }
  if (logits_out) std::memcpy(logits_out, lg.data(), sizeof(float) * m->V);
  return best;
}

void ref_embed(void* hm, const int* tokens, int n, float* out) {
  auto* m = (RefModel*)hm;
  for (int t = 0; t < n; ++t)
    for (int k = 0; k < m->D; ++k) out[(size_t)t * m->D + k] = bf(m->embed[(size_t)tokens[t] * m->D + k]);
}

// generate (pipeline.js:255-281). Returns the number of emitted tokens, -1 on overflow.
int ref_generate(void* hm, const int* tokens, int n, int max_new, int eos, int* out, float* logits) {
  auto* m = (RefModel*)hm;
  std::vector<float> h((size_t)n * m->D);
  ref_embed(hm, tokens, n, h.data());
  if (ref_stage_forward(hm, h.data(), n, 0)) return -1;
  int count = 0;
  int next = ref_sample_last(hm, h.data() + (size_t)(n - 1) * m->D, logits ? logits : nullptr);
  out[count++] = next;
  for (int i = 1; i < max_new; ++i) {
    if (next == eos) break;
    std::vector<float> r(m->D);
    ref_embed(hm, &next, 1, r.data());
    if (ref_stage_forward(hm, r.data(), 1, n + i - 1)) return -1;
    next = ref_sample_last(hm, r.data(), logits ? logits + (size_t)count * m->V : nullptr);
    out[count++] = next;
  }
  return count;
}

}  // extern "C"
