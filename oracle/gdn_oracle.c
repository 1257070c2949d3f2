/*
 * CPU oracle for the Gated DeltaNet recurrence.  TEST INFRASTRUCTURE ONLY: the
 * parity tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it as
 * the checker.  Nothing in the product path (quotebound_b200/) links or calls it.
 *
 * Parity status: UNPINNED against the reference's own bits.  The reference's
 * forward is MLX 0.32.3's closed-over op mx::fast::gated_delta_update and its
 * backward is a Metal kernel (src/delta_grad.cpp:23-145); neither builds on Linux
 * and the reference stores no golden vectors for the recurrence.  This file
 * restates the published algorithm and is cross-checked independently (float64
 * torch autograd and central finite differences, tests/test_oracle.py).
 *
 * Layouts follow the reference (src/deltanet.h:13-16):
 *   q, k [B, T, Hk, Dk]; v, y, dy [B, T, Hv, Dv]; g, beta [B, T, Hv];
 *   state [B, Hv, Dv, Dk] (row r of a value head's state is S[r, :]).
 * Value head hv reads key head hv / (Hv / Hk) (src/delta_grad.cpp:35).
 *
 * Varlen (new in this build; the reference only right-pads, src/data.cpp:24-38):
 * with cu_seqlens (N + 1 int32 offsets) the batch is B = 1 and every sequence
 * n covers steps [cu[n], cu[n+1]); its state starts from h0[n] (or zero) and its
 * final state is hT[n].  Without cu_seqlens, sequence n is batch row n.
 *
 * Accumulation: `acc64` = 1 accumulates every dot product and the state itself in
 * double (a higher-precision oracle); 0 keeps float32 throughout, in the
 * step order of the reference's plain-ops recurrence (tests/gated_delta_ref.h:100-120).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
  int B, T, Hk, Hv, Dk, Dv;
  int N;                 /* number of sequences */
  const int32_t* cu;     /* NULL: fixed-length rows */
} gdn_shape;

static void seq_range(const gdn_shape* s, int n, int64_t* b, int64_t* t0, int64_t* t1) {
  if (s->cu) {
    *b = 0;
    *t0 = s->cu[n];
    *t1 = s->cu[n + 1];
  } else {
    *b = n;
    *t0 = 0;
    *t1 = s->T;
  }
}

static int num_seqs(const gdn_shape* s) { return s->cu ? s->N : s->B; }

/* ---------------------------------------------------------------------------
 * Forward.  Per value head and step (tests/gated_delta_ref.h:110-118):
 *   S = S * g_t;  u = S k_t;  delta = beta_t (v_t - u);  S = S + delta k_t^T;  y_t = S q_t.
 * ------------------------------------------------------------------------- */
#define FWD_BODY(ACC)                                                                           \
  {                                                                                             \
    ACC* S = (ACC*)malloc(sizeof(ACC) * (size_t)Dv * Dk);                                      \
    const size_t s0 = ((size_t)n * Hv + hv) * Dv * Dk;                                         \
    for (size_t i = 0; i < (size_t)Dv * Dk; ++i) S[i] = h0 ? (ACC)h0[s0 + i] : (ACC)0;          \
    for (int64_t t = t0; t < t1; ++t) {                                                         \
      const size_t qk = (((size_t)b * sh->T + t) * Hk + hk) * Dk;                               \
      const size_t vo = (((size_t)b * sh->T + t) * Hv + hv) * Dv;                               \
      const size_t gb = ((size_t)b * sh->T + t) * Hv + hv;                                      \
      const ACC gt = (ACC)g[gb], bt = (ACC)beta[gb];                                            \
      for (int r = 0; r < Dv; ++r) {                                                            \
        ACC* row = S + (size_t)r * Dk;                                                          \
        ACC u = 0;                                                                              \
        for (int i = 0; i < Dk; ++i) {                                                          \
          row[i] = row[i] * gt;                                                                 \
          u += row[i] * (ACC)k[qk + i];                                                         \
        }                                                                                       \
        const ACC d = ((ACC)v[vo + r] - u) * bt;                                                \
        ACC o = 0;                                                                              \
        for (int i = 0; i < Dk; ++i) {                                                          \
          row[i] = row[i] + (ACC)k[qk + i] * d;                                                 \
          o += row[i] * (ACC)q[qk + i];                                                         \
        }                                                                                       \
        y[vo + r] = (float)o;                                                                   \
      }                                                                                         \
    }                                                                                           \
    if (hT)                                                                                     \
      for (size_t i = 0; i < (size_t)Dv * Dk; ++i) hT[s0 + i] = (float)S[i];                    \
    free(S);                                                                                    \
  }

int gdn_oracle_fwd(int B, int T, int Hk, int Hv, int Dk, int Dv, const int32_t* cu, int N, const float* q,
                   const float* k, const float* v, const float* g, const float* beta, const float* h0, float* y,
                   float* hT, int acc64, int threads) {
  if (Hv % Hk) return -1;
  gdn_shape s = {B, T, Hk, Hv, Dk, Dv, N, cu};
  const gdn_shape* sh = &s;
  const int NS = num_seqs(sh);
  const int ratio = Hv / Hk;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic)
#endif
  for (int job = 0; job < NS * Hv; ++job) {
    const int n = job / Hv, hv = job % Hv, hk = hv / ratio;
    int64_t b, t0, t1;
    seq_range(sh, n, &b, &t0, &t1);
    if (acc64)
      FWD_BODY(double)
    else
      FWD_BODY(float)
  }
  return 0;
}

/* ---------------------------------------------------------------------------
 * Backward (src/delta_grad.cpp:13-18, kernel body :97-141).  Chunk-start states
 * every 64 steps are made by the forward itself (:172-181); each chunk is then
 * replayed from its start and walked back.  Going back over step t with dS the
 * cotangent of S:
 *   dS += dy q^T;  dq = S^T dy;  dd = dS k;  dk = dS^T delta;  dv = beta dd;
 *   dbeta = sum(dd (v - u));  du = -beta dd;  dS~ = dS + du k^T;  dk += S~^T du;
 *   dg = sum(dS~ * S_prev);  dS_prev = g dS~.
 * dq and dk are summed over the value heads of a key head in head order (:194-198).
 * ------------------------------------------------------------------------- */
#define CHUNK 64

#define BWD_BODY(ACC)                                                                                 \
  {                                                                                                   \
    const size_t DD = (size_t)Dv * Dk;                                                                \
    const int64_t L = t1 - t0;                                                                        \
    const int64_t NC = (L + CHUNK - 1) / CHUNK;                                                       \
    ACC* ck = (ACC*)malloc(sizeof(ACC) * DD * (size_t)(NC > 0 ? NC : 1));                            \
    ACC* st = (ACC*)malloc(sizeof(ACC) * DD * (CHUNK + 1));                                           \
    ACC* del = (ACC*)malloc(sizeof(ACC) * (size_t)Dv * CHUNK);                                        \
    ACC* uu = (ACC*)malloc(sizeof(ACC) * (size_t)Dv * CHUNK);                                         \
    ACC* ds = (ACC*)malloc(sizeof(ACC) * DD);                                                         \
    ACC* pq = (ACC*)malloc(sizeof(ACC) * Dk);                                                         \
    ACC* pk = (ACC*)malloc(sizeof(ACC) * Dk);                                                         \
    const size_t s0 = ((size_t)n * Hv + hv) * DD;                                                     \
    /* forward to the chunk starts */                                                                 \
    for (size_t i = 0; i < DD; ++i) st[i] = h0 ? (ACC)h0[s0 + i] : (ACC)0;                            \
    for (int64_t c = 0; c < NC; ++c) {                                                                \
      memcpy(ck + (size_t)c * DD, st, sizeof(ACC) * DD);                                              \
      const int64_t a = t0 + c * CHUNK, e = (a + CHUNK < t1) ? a + CHUNK : t1;                        \
      for (int64_t t = a; t < e; ++t) {                                                               \
        const size_t qk = (((size_t)b * sh->T + t) * Hk + hk) * Dk;                                   \
        const size_t vo = (((size_t)b * sh->T + t) * Hv + hv) * Dv;                                   \
        const size_t gb = ((size_t)b * sh->T + t) * Hv + hv;                                          \
        const ACC gt = (ACC)g[gb], bt = (ACC)beta[gb];                                                \
        for (int r = 0; r < Dv; ++r) {                                                                \
          ACC* row = st + (size_t)r * Dk;                                                             \
          ACC u = 0;                                                                                  \
          for (int i = 0; i < Dk; ++i) {                                                              \
            row[i] *= gt;                                                                             \
            u += row[i] * (ACC)k[qk + i];                                                             \
          }                                                                                           \
          const ACC d = ((ACC)v[vo + r] - u) * bt;                                                    \
          for (int i = 0; i < Dk; ++i) row[i] += (ACC)k[qk + i] * d;                                  \
        }                                                                                             \
      }                                                                                               \
    }                                                                                                 \
    for (size_t i = 0; i < DD; ++i) ds[i] = dhT ? (ACC)dhT[s0 + i] : (ACC)0;                          \
    for (int64_t c = NC - 1; c >= 0; --c) {                                                           \
      const int64_t a = t0 + c * CHUNK, e = (a + CHUNK < t1) ? a + CHUNK : t1;                        \
      memcpy(st, ck + (size_t)c * DD, sizeof(ACC) * DD);                                              \
      for (int64_t t = a; t < e; ++t) { /* replay, keeping every state of the chunk */                \
        const int64_t j = t - a;                                                                      \
        const size_t qk = (((size_t)b * sh->T + t) * Hk + hk) * Dk;                                   \
        const size_t vo = (((size_t)b * sh->T + t) * Hv + hv) * Dv;                                   \
        const size_t gb = ((size_t)b * sh->T + t) * Hv + hv;                                          \
        const ACC gt = (ACC)g[gb], bt = (ACC)beta[gb];                                                \
        ACC* prev = st + (size_t)j * DD;                                                              \
        ACC* next = st + (size_t)(j + 1) * DD;                                                        \
        for (int r = 0; r < Dv; ++r) {                                                                \
          ACC u = 0;                                                                                  \
          for (int i = 0; i < Dk; ++i) {                                                              \
            next[(size_t)r * Dk + i] = prev[(size_t)r * Dk + i] * gt;                                 \
            u += next[(size_t)r * Dk + i] * (ACC)k[qk + i];                                           \
          }                                                                                           \
          const ACC d = ((ACC)v[vo + r] - u) * bt;                                                    \
          for (int i = 0; i < Dk; ++i) next[(size_t)r * Dk + i] += (ACC)k[qk + i] * d;                \
          del[(size_t)j * Dv + r] = d;                                                                \
          uu[(size_t)j * Dv + r] = u;                                                                 \
        }                                                                                             \
      }                                                                                               \
      for (int64_t t = e - 1; t >= a; --t) {                                                          \
        const int64_t j = t - a;                                                                      \
        const size_t qk = (((size_t)b * sh->T + t) * Hk + hk) * Dk;                                   \
        const size_t vo = (((size_t)b * sh->T + t) * Hv + hv) * Dv;                                   \
        const size_t gb = ((size_t)b * sh->T + t) * Hv + hv;                                          \
        const ACC gt = (ACC)g[gb], bt = (ACC)beta[gb];                                                \
        const ACC* Sp = st + (size_t)j * DD;       /* S_{t-1} */                                      \
        const ACC* Sn = st + (size_t)(j + 1) * DD; /* S_t */                                          \
        for (int i = 0; i < Dk; ++i) pq[i] = pk[i] = 0;                                               \
        ACC dgs = 0, dbs = 0;                                                                         \
        for (int r = 0; r < Dv; ++r) {                                                                \
          ACC* dr = ds + (size_t)r * Dk;                                                              \
          const ACC dyr = (ACC)dy[vo + r];                                                            \
          ACC dd = 0;                                                                                 \
          for (int i = 0; i < Dk; ++i) {                                                              \
            dr[i] += dyr * (ACC)q[qk + i];                                                            \
            pq[i] += dyr * Sn[(size_t)r * Dk + i];                                                    \
            dd += dr[i] * (ACC)k[qk + i];                                                             \
          }                                                                                           \
          const ACC du = -bt * dd;                                                                    \
          const ACC dl = del[(size_t)j * Dv + r];                                                     \
          ACC dgr = 0;                                                                                \
          for (int i = 0; i < Dk; ++i) {                                                              \
            pk[i] += dr[i] * dl + du * (Sp[(size_t)r * Dk + i] * gt);                                 \
            dr[i] += du * (ACC)k[qk + i];                                                             \
            dgr += dr[i] * Sp[(size_t)r * Dk + i];                                                    \
            dr[i] *= gt;                                                                              \
          }                                                                                           \
          dv[vo + r] = (float)(bt * dd);                                                              \
          dbs += dd * ((ACC)v[vo + r] - uu[(size_t)j * Dv + r]);                                      \
          dgs += dgr;                                                                                 \
        }                                                                                             \
        const size_t pp = ((((size_t)b * sh->T + t) * Hv) + hv) * Dk;                                 \
        for (int i = 0; i < Dk; ++i) {                                                                \
          dq_part[pp + i] = (double)pq[i];                                                            \
          dk_part[pp + i] = (double)pk[i];                                                            \
        }                                                                                             \
        dg[gb] = (float)dgs;                                                                          \
        dbeta[gb] = (float)dbs;                                                                       \
      }                                                                                               \
    }                                                                                                 \
    if (dh0)                                                                                          \
      for (size_t i = 0; i < DD; ++i) dh0[s0 + i] = (float)ds[i];                                     \
    free(ck);                                                                                         \
    free(st);                                                                                         \
    free(del);                                                                                        \
    free(uu);                                                                                         \
    free(ds);                                                                                         \
    free(pq);                                                                                         \
    free(pk);                                                                                         \
  }

int gdn_oracle_bwd(int B, int T, int Hk, int Hv, int Dk, int Dv, const int32_t* cu, int N, const float* q,
                   const float* k, const float* v, const float* g, const float* beta, const float* h0,
                   const float* dy, const float* dhT, float* dq, float* dk, float* dv, float* dg, float* dbeta,
                   float* dh0, int acc64, int threads) {
  if (Hv % Hk) return -1;
  gdn_shape s = {B, T, Hk, Hv, Dk, Dv, N, cu};
  const gdn_shape* sh = &s;
  const int NS = num_seqs(sh);
  const int ratio = Hv / Hk;
  /* per value head dq/dk rows, summed over the group afterwards in head order */
  const size_t parts = (size_t)B * T * Hv * Dk;
  double* dq_part = (double*)calloc(parts, sizeof(double));
  double* dk_part = (double*)calloc(parts, sizeof(double));
  if (!dq_part || !dk_part) {
    free(dq_part);
    free(dk_part);
    return -2;
  }
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic)
#endif
  for (int job = 0; job < NS * Hv; ++job) {
    const int n = job / Hv, hv = job % Hv, hk = hv / ratio;
    int64_t b, t0, t1;
    seq_range(sh, n, &b, &t0, &t1);
    if (acc64)
      BWD_BODY(double)
    else
      BWD_BODY(float)
  }
#ifdef _OPENMP
#pragma omp parallel for
#endif
  for (int64_t bt = 0; bt < (int64_t)B * T; ++bt)
    for (int hk = 0; hk < Hk; ++hk)
      for (int i = 0; i < Dk; ++i) {
        double aq = 0, ak = 0;
        for (int j = 0; j < ratio; ++j) {
          const size_t pp = ((size_t)bt * Hv + hk * ratio + j) * Dk + i;
          aq += dq_part[pp];
          ak += dk_part[pp];
        }
        dq[((size_t)bt * Hk + hk) * Dk + i] = (float)aq;
        dk[((size_t)bt * Hk + hk) * Dk + i] = (float)ak;
      }
  free(dq_part);
  free(dk_part);
  return 0;
}

/* ---------------------------------------------------------------------------
 * Gate, beta and q/k norm (src/deltanet.cpp:22-33 compute_g, :94-100).
 *   qn = q * rsqrt(mean(q^2) + 1e-6) * (1/Dk);  kn = k * rsqrt(mean(k^2) + 1e-6) * (1/sqrt(Dk));
 *   beta = sigmoid(b);  g = exp(-exp(A_log) * softplus(a + dt_bias)),  softplus(x) = logaddexp(x, 0).
 * Computed in double, returned as float.  q, k [M, Dk] rows (M = B*T*Hk); a, b [P, Hv] (P = B*T).
 * ------------------------------------------------------------------------- */
static double softplus_d(double x) { return x > 0 ? x + log1p(exp(-x)) : log1p(exp(x)); }
static double sigmoid_d(double x) { return 1.0 / (1.0 + exp(-x)); }

int gdn_oracle_gate_fwd(int64_t M, int Dk, int64_t P, int Hv, const float* q, const float* k, const float* a,
                        const float* b, const float* A_log, const float* dt_bias, float* qn, float* kn, float* g,
                        float* beta, float* logg) {
  const double sq = 1.0 / Dk, sk = 1.0 / sqrt((double)Dk);
  for (int64_t m = 0; m < M; ++m) {
    double sq2 = 0, sk2 = 0;
    for (int i = 0; i < Dk; ++i) {
      sq2 += (double)q[m * Dk + i] * q[m * Dk + i];
      sk2 += (double)k[m * Dk + i] * k[m * Dk + i];
    }
    const double rq = 1.0 / sqrt(sq2 / Dk + 1e-6), rk = 1.0 / sqrt(sk2 / Dk + 1e-6);
    for (int i = 0; i < Dk; ++i) {
      qn[m * Dk + i] = (float)(q[m * Dk + i] * rq * sq);
      kn[m * Dk + i] = (float)(k[m * Dk + i] * rk * sk);
    }
  }
  for (int64_t p = 0; p < P; ++p)
    for (int h = 0; h < Hv; ++h) {
      const double x = (double)a[p * Hv + h] + dt_bias[h];
      const double lg = -exp((double)A_log[h]) * softplus_d(x);
      g[p * Hv + h] = (float)exp(lg);
      if (logg) logg[p * Hv + h] = (float)lg;
      beta[p * Hv + h] = (float)sigmoid_d(b[p * Hv + h]);
    }
  return 0;
}

/* Chain rule of the above given the recurrence's cotangents dqn, dkn [M, Dk], dg, dbeta [P, Hv].
 * dA_log[h] = sum dg g (-e^A softplus(x)); ddt_bias[h] = sum dg g (-e^A sigmoid(x)); da = the same per element. */
int gdn_oracle_gate_bwd(int64_t M, int Dk, int64_t P, int Hv, const float* q, const float* k, const float* a,
                        const float* b, const float* A_log, const float* dt_bias, const float* dqn,
                        const float* dkn, const float* dg, const float* dbeta, float* dq, float* dk, float* da,
                        float* db, float* dA_log, float* ddt_bias) {
  const double sq = 1.0 / Dk, sk = 1.0 / sqrt((double)Dk);
  for (int64_t m = 0; m < M; ++m) {
    double q2 = 0, k2 = 0, qd = 0, kd = 0;
    for (int i = 0; i < Dk; ++i) {
      const double qi = q[m * Dk + i], ki = k[m * Dk + i];
      q2 += qi * qi;
      k2 += ki * ki;
      qd += qi * dqn[m * Dk + i];
      kd += ki * dkn[m * Dk + i];
    }
    const double rq = 1.0 / sqrt(q2 / Dk + 1e-6), rk = 1.0 / sqrt(k2 / Dk + 1e-6);
    for (int i = 0; i < Dk; ++i) {
      dq[m * Dk + i] = (float)(sq * (rq * dqn[m * Dk + i] - rq * rq * rq * qd * q[m * Dk + i] / Dk));
      dk[m * Dk + i] = (float)(sk * (rk * dkn[m * Dk + i] - rk * rk * rk * kd * k[m * Dk + i] / Dk));
    }
  }
  for (int h = 0; h < Hv; ++h) {
    double sa = 0, sd = 0;
    const double eA = exp((double)A_log[h]);
    for (int64_t p = 0; p < P; ++p) {
      const double x = (double)a[p * Hv + h] + dt_bias[h];
      const double lg = -eA * softplus_d(x);
      const double dl = (double)dg[p * Hv + h] * exp(lg); /* d loss / d log g */
      const double dx = dl * (-eA * sigmoid_d(x));
      da[p * Hv + h] = (float)dx;
      sd += dx;
      sa += dl * lg;
      const double bb = sigmoid_d(b[p * Hv + h]);
      db[p * Hv + h] = (float)(dbeta[p * Hv + h] * bb * (1 - bb));
    }
    dA_log[h] = (float)sa;
    ddt_bias[h] = (float)sd;
  }
  return 0;
}


/* ---------------------------------------------------------------------------
 * Around the recurrence.  round_bf16 = 1 rounds what the reference keeps in the activations' dtype
 * (bf16): the conv's output before its SiLU and the SiLU's output; the norm's output before the gate
 * and the gated output.  Everything else in double.
 * ------------------------------------------------------------------------- */
static float bf16_round(float x) { /* round to nearest even at 8 mantissa bits */
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  memcpy(&x, &u, 4);
  return x;
}
static double rnd(double x, int round_bf16) { return round_bf16 ? (double)bf16_round((float)x) : (double)(float)x; }

/* The causal depthwise conv1d + SiLU (src/deltanet.cpp:74-93): per sequence n, xpad = [state_in[n]
 * (K - 1 rows; zeros when NULL); its x rows], u_t[c] = sum_m xpad[t + m][c] w[c][m], y = silu(u),
 * split into q | k | v by channel; state_out[n] = the last K - 1 rows of xpad (src/deltanet.cpp:75-77).
 * x [tokens, conv_dim] with conv_dim = 2 key_dim + value_dim; w [conv_dim, K]. */
static void conv_seq(const gdn_shape* s, int n, int64_t* t0, int64_t* t1) {
  int64_t b;
  seq_range(s, n, &b, t0, t1);
  if (!s->cu) { *t0 = (int64_t)n * s->T; *t1 = *t0 + s->T; }
}

int gdn_oracle_conv_fwd(int B, int T, const int32_t* cu, int N, int key_dim, int value_dim, int K, int round_bf16,
                        const float* x, const float* w, const float* state_in, float* q, float* k, float* v,
                        float* state_out) {
  const gdn_shape sh = {B, T, 1, 1, 1, 1, N, cu};
  const int cd = 2 * key_dim + value_dim, NS = num_seqs(&sh);
  for (int n = 0; n < NS; ++n) {
    int64_t t0, t1;
    conv_seq(&sh, n, &t0, &t1);
    const int64_t Ls = t1 - t0;
    for (int c = 0; c < cd; ++c) {
      /* xpad value at padded position p */
#define XPAD(p) ((p) < K - 1 ? (state_in ? (double)state_in[((int64_t)n * (K - 1) + (p)) * cd + c] : 0.0) \
                             : (double)x[(t0 + (p) - (K - 1)) * cd + c])
      for (int64_t t = 0; t < Ls; ++t) {
        double u = 0;
        for (int m = 0; m < K; ++m) u += XPAD(t + m) * (double)w[(int64_t)c * K + m];
        u = rnd(u, round_bf16);
        const float y = (float)rnd(u / (1.0 + exp(-u)), round_bf16);
        const int64_t tok = t0 + t;
        if (c < key_dim) q[tok * key_dim + c] = y;
        else if (c < 2 * key_dim) k[tok * key_dim + c - key_dim] = y;
        else v[tok * value_dim + c - 2 * key_dim] = y;
      }
      if (state_out)
        for (int j = 0; j < K - 1; ++j) state_out[((int64_t)n * (K - 1) + j) * cd + c] = (float)XPAD(Ls + j);
#undef XPAD
    }
  }
  return 0;
}

/* Its backward: du = dy silu'(u) (u rounded as in the forward; a rounding passes the cotangent
 * through), dxpad[t + m] += du_t w[m], dw[c][m] += du_t xpad[t + m]; the new state's cotangent adds onto
 * xpad's last K - 1 rows; xpad's first K - 1 rows are the carried state's cotangent. */
int gdn_oracle_conv_bwd(int B, int T, const int32_t* cu, int N, int key_dim, int value_dim, int K, int round_bf16,
                        const float* x, const float* w, const float* state_in, const float* dq, const float* dk,
                        const float* dv, const float* dstate_out, float* dx, float* dw, float* dstate_in) {
  const gdn_shape sh = {B, T, 1, 1, 1, 1, N, cu};
  const int cd = 2 * key_dim + value_dim, NS = num_seqs(&sh);
  double* dwa = (double*)calloc((size_t)cd * K, sizeof(double));
  for (int n = 0; n < NS; ++n) {
    int64_t t0, t1;
    conv_seq(&sh, n, &t0, &t1);
    const int64_t Ls = t1 - t0;
    double* dxp = (double*)malloc(sizeof(double) * (size_t)(Ls + K - 1));
    for (int c = 0; c < cd; ++c) {
#define XPAD(p) ((p) < K - 1 ? (state_in ? (double)state_in[((int64_t)n * (K - 1) + (p)) * cd + c] : 0.0) \
                             : (double)x[(t0 + (p) - (K - 1)) * cd + c])
      for (int64_t p = 0; p < Ls + K - 1; ++p) dxp[p] = 0;
      for (int64_t t = 0; t < Ls; ++t) {
        double u = 0;
        for (int m = 0; m < K; ++m) u += XPAD(t + m) * (double)w[(int64_t)c * K + m];
        u = rnd(u, round_bf16);
        const int64_t tok = t0 + t;
        const double g = c < key_dim ? dq[tok * key_dim + c]
                         : c < 2 * key_dim ? dk[tok * key_dim + c - key_dim]
                                           : dv[tok * value_dim + c - 2 * key_dim];
        const double sg = 1.0 / (1.0 + exp(-u));
        const double du = g * sg * (1.0 + u * (1.0 - sg));
        for (int m = 0; m < K; ++m) {
          dxp[t + m] += du * w[(int64_t)c * K + m];
          dwa[(int64_t)c * K + m] += du * XPAD(t + m);
        }
      }
      if (dstate_out)
        for (int j = 0; j < K - 1; ++j) dxp[Ls + j] += dstate_out[((int64_t)n * (K - 1) + j) * cd + c];
      for (int64_t p = 0; p < Ls + K - 1; ++p) {
        if (p < K - 1) {
          if (dstate_in) dstate_in[((int64_t)n * (K - 1) + p) * cd + c] = (float)dxp[p];
        } else {
          dx[(t0 + p - (K - 1)) * cd + c] = (float)dxp[p];
        }
      }
#undef XPAD
    }
    free(dxp);
  }
  if (dw)
    for (int64_t i = 0; i < (int64_t)cd * K; ++i) dw[i] = (float)dwa[i];
  free(dwa);
  return 0;
}

/* The gated RMSNorm (src/deltanet.cpp:35-45, :122): per row of Dv, n = y rsqrt(mean(y^2) + eps) w
 * (rounded), o = silu(z) n (rounded). */
int gdn_oracle_gated_norm_fwd(int64_t rows, int Dv, float eps, int round_bf16, const float* y, const float* z,
                              const float* w, float* o) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* yr = y + r * Dv;
    double ss = 0;
    for (int i = 0; i < Dv; ++i) ss += (double)yr[i] * yr[i];
    const double rs = 1.0 / sqrt(ss / Dv + eps);
    for (int i = 0; i < Dv; ++i) {
      const double nv = rnd(yr[i] * rs * w[i], round_bf16);
      const double zz = z[r * Dv + i];
      o[r * Dv + i] = (float)rnd(zz / (1.0 + exp(-zz)) * nv, round_bf16);
    }
  }
  return 0;
}

int gdn_oracle_gated_norm_bwd(int64_t rows, int Dv, float eps, int round_bf16, const float* y, const float* z,
                              const float* w, const float* dout, float* dy, float* dz, float* dw) {
  double* dwa = (double*)calloc((size_t)Dv, sizeof(double));
  for (int64_t r = 0; r < rows; ++r) {
    const float* yr = y + r * Dv;
    double ss = 0, dot = 0;
    for (int i = 0; i < Dv; ++i) ss += (double)yr[i] * yr[i];
    const double rs = 1.0 / sqrt(ss / Dv + eps);
    for (int i = 0; i < Dv; ++i) {
      const double zz = z[r * Dv + i], sg = 1.0 / (1.0 + exp(-zz));
      const double nv = rnd(yr[i] * rs * w[i], round_bf16);
      const double g = dout[r * Dv + i], dn = g * zz * sg;
      dz[r * Dv + i] = (float)(g * nv * sg * (1.0 + zz * (1.0 - sg)));
      dot += (double)yr[i] * w[i] * dn;
      dwa[i] += dn * yr[i] * rs;
    }
    for (int i = 0; i < Dv; ++i) {
      const double zz = z[r * Dv + i], sg = 1.0 / (1.0 + exp(-zz));
      const double dn = (double)dout[r * Dv + i] * zz * sg;
      dy[r * Dv + i] = (float)(rs * w[i] * dn - rs * rs * rs * dot * yr[i] / Dv);
    }
  }
  if (dw)
    for (int i = 0; i < Dv; ++i) dw[i] = (float)dwa[i];
  free(dwa);
  return 0;
}

int gdn_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
