/*
 * CPU restatement of Expert Sniper's MoE block in C (fp32, pthreads).
 *
 * TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and bench.py's
 * CPU baseline / reference arm load this library as the checker or as the
 * timed CPU implementation. The product (expert_sniper_b200) never links it.
 *
 * Restates, with the same arithmetic as oracle/moe_oracle.py:
 *   oracle_route       src/mlx_expert_sniper/generate.py:122-136 (bias add,
 *                      fp32 softmax, top-k with lower-id tie break,
 *                      renormalisation)
 *   oracle_expert_ffn  src/mlx_expert_sniper/engine.py:15-42 run_expert_ffn
 *                      (dequant w = scale*q + bias per 64-group, gate/up,
 *                      silu(g)*u, down, weighted sum over the k slots in
 *                      ascending expert id order), the shared expert of
 *                      generate.py:173-178, and the -1 partition mask of
 *                      src/expert_network/node.py:142-172.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <pthread.h>
#include <string.h>
#include <unistd.h>

/* ---- a minimal parallel-for over [0, n) with dynamic chunks of 1 -------- */
typedef void (*body_fn)(void* ctx, int i);
typedef struct {
  body_fn fn;
  void* ctx;
  int n;
  int next;
  pthread_mutex_t mu;
} pfor_state;

static void* pfor_worker(void* arg) {
  pfor_state* st = (pfor_state*)arg;
  for (;;) {
    pthread_mutex_lock(&st->mu);
    const int i = st->next++;
    pthread_mutex_unlock(&st->mu);
    if (i >= st->n) break;
    st->fn(st->ctx, i);
  }
  return NULL;
}

static int g_threads = 0;

static void parallel_for(int n, body_fn fn, void* ctx) {
  int nt = g_threads > 0 ? g_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nt < 1) nt = 1;
  if (nt > n) nt = n;
  pfor_state st = {fn, ctx, n, 0, PTHREAD_MUTEX_INITIALIZER};
  if (nt <= 1) {
    pfor_worker(&st);
    return;
  }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
  for (int i = 0; i < nt; ++i) pthread_create(&th[i], NULL, pfor_worker, &st);
  for (int i = 0; i < nt; ++i) pthread_join(th[i], NULL);
  free(th);
}

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: man * 2^-24 */
      float f = (float)man * (1.0f / 16777216.0f);
      return (h & 0x8000u) ? -f : f;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

typedef struct {
  const float* logits;
  const float* bias;
  int E, k, renorm;
  int32_t* idx;
  float* w;
} route_ctx;

static void route_one(void* vctx, int t) {
  const route_ctx* c = (const route_ctx*)vctx;
  const int E = c->E, k = c->k;
  const float* l = c->logits + (size_t)t * E;
  float* z = (float*)malloc(sizeof(float) * E);
  char* taken = (char*)calloc(E, 1);
  float m = -INFINITY;
  for (int e = 0; e < E; ++e) {
    z[e] = l[e] + (c->bias ? c->bias[e] : 0.f);
    if (z[e] > m) m = z[e];
  }
  double s = 0.0;
  for (int e = 0; e < E; ++e) s += expf(z[e] - m);
  float tot = 0.f;
  for (int j = 0; j < k; ++j) {
    int best = -1;
    for (int e = 0; e < E; ++e)
      if (!taken[e] && (best < 0 || z[e] > z[best])) best = e;
    taken[best] = 1;
    c->idx[(size_t)t * k + j] = best;
    c->w[(size_t)t * k + j] = (float)(expf(z[best] - m) / s);
    tot += c->w[(size_t)t * k + j];
  }
  if (c->renorm)
    for (int j = 0; j < k; ++j) c->w[(size_t)t * k + j] /= tot;
  free(z);
  free(taken);
}

int oracle_route(const float* logits, const float* bias, int T, int E, int k, int renorm,
                 int32_t* idx, float* w) {
  if (T < 0 || E <= 0 || k <= 0 || k > E) return 1;
  route_ctx c = {logits, bias, E, k, renorm, idx, w};
  parallel_for(T, route_one, &c);
  return 0;
}

/* y[n][r] = sum_k dequant(W)[r][k] * X[n][k] for the listed tokens. */
static void qgemv_rows(const uint32_t* wq, const uint16_t* ws, const uint16_t* wb, int N, int K,
                       const float* X, int ntok, float* Y /* [ntok][N] */) {
  float deq[64];
  for (int r = 0; r < N; ++r) {
    const uint32_t* row = wq + (size_t)r * (K / 8);
    for (int n = 0; n < ntok; ++n) Y[(size_t)n * N + r] = 0.f;
    for (int g = 0; g < K / 64; ++g) {
      const float s = half_to_float(ws[(size_t)r * (K / 64) + g]);
      const float b = half_to_float(wb[(size_t)r * (K / 64) + g]);
      for (int i = 0; i < 64; ++i) {
        const uint32_t word = row[g * 8 + (i >> 3)];
        deq[i] = s * (float)((word >> (4 * (i & 7))) & 0xfu) + b;
      }
      for (int n = 0; n < ntok; ++n) {
        const float* xv = X + (size_t)n * K + g * 64;
        float acc = 0.f;
        for (int i = 0; i < 64; ++i) acc += deq[i] * xv[i];
        Y[(size_t)n * N + r] += acc;
      }
    }
  }
}

typedef struct {
  const uint32_t* w[3];
  const uint16_t* s[3];
  const uint16_t* b[3];
} proj3;

/* out[n] = down(silu(gate(X_n)) * up(X_n)) for ntok tokens. */
static void swiglu_expert(const proj3* p, size_t eoff_gu_w, size_t eoff_gu_s, size_t eoff_d_w,
                          size_t eoff_d_s, int D, int I, const float* X, int ntok, float* out) {
  float* g = (float*)malloc(sizeof(float) * (size_t)ntok * I);
  float* u = (float*)malloc(sizeof(float) * (size_t)ntok * I);
  qgemv_rows(p->w[0] + eoff_gu_w, p->s[0] + eoff_gu_s, p->b[0] + eoff_gu_s, I, D, X, ntok, g);
  qgemv_rows(p->w[1] + eoff_gu_w, p->s[1] + eoff_gu_s, p->b[1] + eoff_gu_s, I, D, X, ntok, u);
  for (size_t i = 0; i < (size_t)ntok * I; ++i) {
    const float gv = g[i];
    g[i] = gv / (1.f + expf(-gv)) * u[i];
  }
  qgemv_rows(p->w[2] + eoff_d_w, p->s[2] + eoff_d_s, p->b[2] + eoff_d_s, D, I, g, ntok, out);
  free(g);
  free(u);
}

typedef struct {
  const proj3* p;
  const float* x;
  int T, D, I, k;
  const int32_t* idx;
  float* y;
} expert_ctx;

static void expert_one(void* vctx, int e) {
  const expert_ctx* c = (const expert_ctx*)vctx;
  const int T = c->T, D = c->D, I = c->I, k = c->k;
  int ntok = 0;
  for (int i = 0; i < T * k; ++i) ntok += c->idx[i] == e;
  if (!ntok) return;
  int* slot = (int*)malloc(sizeof(int) * ntok);
  float* X = (float*)malloc(sizeof(float) * (size_t)ntok * D);
  float* Y = (float*)malloc(sizeof(float) * (size_t)ntok * D);
  int n = 0;
  for (int i = 0; i < T * k; ++i)
    if (c->idx[i] == e) {
      slot[n] = i;
      memcpy(X + (size_t)n * D, c->x + (size_t)(i / k) * D, sizeof(float) * D);
      ++n;
    }
  swiglu_expert(c->p, (size_t)e * I * (D / 8), (size_t)e * I * (D / 64), (size_t)e * D * (I / 8),
                (size_t)e * D * (I / 64), D, I, X, ntok, Y);
  for (int m = 0; m < ntok; ++m)
    memcpy(c->y + (size_t)slot[m] * D, Y + (size_t)m * D, sizeof(float) * D);
  free(slot);
  free(X);
  free(Y);
}

typedef struct {
  const int32_t* idx;
  const float* w;
  const float* y;
  float* out;
  int D, k;
} combine_ctx;

static void combine_one(void* vctx, int t) {
  const combine_ctx* c = (const combine_ctx*)vctx;
  const int D = c->D, k = c->k;
  float* o = c->out + (size_t)t * D;
  for (int d = 0; d < D; ++d) o[d] = 0.f;
  /* slots in ascending expert id order (stable on equal ids) */
  int order[64];
  int m = 0;
  for (int j = 0; j < k && j < 64; ++j) {
    const int e = c->idx[(size_t)t * k + j];
    if (e < 0) continue;
    int i = m++;
    while (i > 0 && c->idx[(size_t)t * k + order[i - 1]] > e) {
      order[i] = order[i - 1];
      --i;
    }
    order[i] = j;
  }
  for (int i = 0; i < m; ++i) {
    const int j = order[i];
    const float wj = c->w[(size_t)t * k + j];
    const float* yv = c->y + ((size_t)t * k + j) * D;
    for (int d = 0; d < D; ++d) o[d] += wj * yv[d];
  }
}

typedef struct {
  const proj3* p;
  const float* x;
  float* Y;
  int T, D, I, chunk;
} shared_ctx;

static void shared_one(void* vctx, int ci) {
  const shared_ctx* c = (const shared_ctx*)vctx;
  const int t0 = ci * c->chunk;
  const int nt = (c->T - t0) < c->chunk ? (c->T - t0) : c->chunk;
  swiglu_expert(c->p, 0, 0, 0, 0, c->D, c->I, c->x + (size_t)t0 * c->D, nt, c->Y + (size_t)t0 * c->D);
}

int oracle_expert_ffn(const float* x, int T, int D, int I, int E, int k,
                      const uint32_t* gw, const uint16_t* gs, const uint16_t* gb,
                      const uint32_t* uw, const uint16_t* us, const uint16_t* ub,
                      const uint32_t* dw, const uint16_t* ds, const uint16_t* db,
                      const uint32_t* sgw_, const uint16_t* sgs, const uint16_t* sgb,
                      const uint32_t* suw, const uint16_t* sus, const uint16_t* sub,
                      const uint32_t* sdw, const uint16_t* sds, const uint16_t* sdb,
                      const float* shared_gate_w, const int32_t* idx, const float* w,
                      float* out, int nthreads) {
  if (T < 0 || D % 64 || I % 64 || k <= 0 || k > 64) return 1;
  g_threads = nthreads;
  proj3 p = {{gw, uw, dw}, {gs, us, ds}, {gb, ub, db}};
  float* y = (float*)calloc((size_t)T * k * D + 1, sizeof(float));
  if (!y) return 2;
  expert_ctx ec = {&p, x, T, D, I, k, idx, y};
  parallel_for(E, expert_one, &ec);
  combine_ctx cc = {idx, w, y, out, D, k};
  parallel_for(T, combine_one, &cc);
  free(y);
  if (sgw_) {
    proj3 sp = {{sgw_, suw, sdw}, {sgs, sus, sds}, {sgb, sub, sdb}};
    float* Y = (float*)malloc(sizeof(float) * ((size_t)T * D + 1));
    shared_ctx sc = {&sp, x, Y, T, D, I, 16};
    parallel_for((T + 15) / 16, shared_one, &sc);
    for (int t = 0; t < T; ++t) {
      float gate = 1.f;
      if (shared_gate_w) {
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot += x[(size_t)t * D + d] * shared_gate_w[d];
        gate = 1.f / (1.f + expf(-dot));
      }
      for (int d = 0; d < D; ++d) out[(size_t)t * D + d] += gate * Y[(size_t)t * D + d];
    }
    free(Y);
  }
  g_threads = 0;
  return 0;
}
