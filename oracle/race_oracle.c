/*
 * race_oracle.c -- CPU oracle for the causal RACE attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
 * legs may load it.  The CUDA library (race_attention_b200/csrc) never calls it
 * and the Python operator surface fails loudly instead of falling back to it.
 *
 * It restates, in plain C with double-precision accumulation, the reference's
 * own algorithm (paths relative to the reference project root):
 *
 *   oracle_soft_hash      scaling/race_common.py:36-73   (soft_hash_probs)
 *   oracle_soft_hash_bwd  autograd of scaling/race_common.py:56-72
 *   oracle_race_fwd       scaling/race_common.py:76-90   (race_prefix_ref),
 *                         extended with an optional carried-in state (A0,B0)
 *                         so the same routine is the decode-step and the
 *                         sequence-shard oracle
 *   oracle_race_bwd       scaling/race_causal_cpu.py:52-72 composed with
 *                         kernels/cpu/race_pref.cpp:104-220
 *                         (race_prefix_mean_flat_bw), restated per (n,s)
 *                         stream without materialising V expanded x S, and
 *                         extended with an incoming suffix gradient (gA, gB)
 *                         for the final state, which is what a later sequence
 *                         shard sends back to an earlier one
 *
 * Layouts are the reference's: Q/K/V/out [N,T,D]; probs [N,T,S] with
 * S = L*R, R = 2^P, bucket index s = l*R + r (table-outer, corner-inner);
 * planes_T [D, L*P] with column j = l*P + p; corner r has hyperplane sign
 * +1 for bit p iff bit (P-1-p) of r is set (itertools.product order,
 * scaling/race_common.py:30-32).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

int oracle_abi_version(void) { return 1; }

static inline double corner_sign(long r, long p, long P)
{
    return ((r >> (P - 1 - p)) & 1) ? 1.0 : -1.0;
}

/* probs[n,t,l*R+r] = softmax_r( sum_p tanh(x.planes_T[:,l*P+p]) * scale * sign(p,r) ) */
void oracle_soft_hash(const double *X, long N, long T, long D,
                      const double *planes_T, long L, long P, double logit_scale,
                      double *probs)
{
    const long LP = L * P, R = 1L << P, S = L * R;
    double *a = (double *)malloc(sizeof(double) * LP);
    double *lg = (double *)malloc(sizeof(double) * R);
    for (long n = 0; n < N; ++n)
        for (long t = 0; t < T; ++t) {
            const double *x = X + (n * T + t) * D;
            double *pr = probs + (n * T + t) * S;
            for (long j = 0; j < LP; ++j) {
                double acc = 0.0;
                for (long d = 0; d < D; ++d) acc += x[d] * planes_T[d * LP + j];
                a[j] = tanh(acc) * logit_scale;
            }
            for (long l = 0; l < L; ++l) {
                double mx = -INFINITY;
                for (long r = 0; r < R; ++r) {
                    double v = 0.0;
                    for (long p = 0; p < P; ++p) v += a[l * P + p] * corner_sign(r, p, P);
                    lg[r] = v;
                    if (v > mx) mx = v;
                }
                double z = 0.0;
                for (long r = 0; r < R; ++r) { lg[r] = exp(lg[r] - mx); z += lg[r]; }
                for (long r = 0; r < R; ++r) pr[l * R + r] = lg[r] / z;
            }
        }
    free(a);
    free(lg);
}

/* dX = d/dX < dprobs, soft_hash(X) >  (planes are buffers: no gradient for them). */
void oracle_soft_hash_bwd(const double *X, long N, long T, long D,
                          const double *planes_T, long L, long P, double logit_scale,
                          const double *dprobs, double *dX)
{
    const long LP = L * P, R = 1L << P, S = L * R;
    double *th = (double *)malloc(sizeof(double) * LP);
    double *da = (double *)malloc(sizeof(double) * LP);
    double *pr = (double *)malloc(sizeof(double) * R);
    for (long n = 0; n < N; ++n)
        for (long t = 0; t < T; ++t) {
            const double *x = X + (n * T + t) * D;
            const double *g = dprobs + (n * T + t) * S;
            double *dx = dX + (n * T + t) * D;
            for (long j = 0; j < LP; ++j) {
                double acc = 0.0;
                for (long d = 0; d < D; ++d) acc += x[d] * planes_T[d * LP + j];
                th[j] = tanh(acc);
            }
            for (long l = 0; l < L; ++l) {
                double mx = -INFINITY;
                for (long r = 0; r < R; ++r) {
                    double v = 0.0;
                    for (long p = 0; p < P; ++p) v += th[l * P + p] * logit_scale * corner_sign(r, p, P);
                    pr[r] = v;
                    if (v > mx) mx = v;
                }
                double z = 0.0;
                for (long r = 0; r < R; ++r) { pr[r] = exp(pr[r] - mx); z += pr[r]; }
                double c = 0.0;
                for (long r = 0; r < R; ++r) { pr[r] /= z; c += pr[r] * g[l * R + r]; }
                for (long p = 0; p < P; ++p) {
                    double acc = 0.0;
                    for (long r = 0; r < R; ++r)
                        acc += pr[r] * (g[l * R + r] - c) * corner_sign(r, p, P);
                    da[l * P + p] = acc;
                }
            }
            for (long d = 0; d < D; ++d) {
                double acc = 0.0;
                for (long j = 0; j < LP; ++j)
                    acc += da[j] * logit_scale * (1.0 - th[j] * th[j]) * planes_T[d * LP + j];
                dx[d] = acc;
            }
        }
    free(th);
    free(da);
    free(pr);
}

/*
 * out[n,t,:] = sum_s pq[n,t,s] * B_t[n,s,:] / (A_t[n,s] + eps)
 * A_t = A0 + sum_{tau<=t} pk[tau],  B_t = B0 + sum_{tau<=t} pk[tau] * V[tau]
 * A0/B0 may be NULL (zero state).  A_fin/B_fin may be NULL.
 */
void oracle_race_fwd(const double *pk, const double *pq, const double *V,
                     long N, long T, long S, long D, double eps,
                     const double *A0, const double *B0,
                     double *out, double *A_fin, double *B_fin)
{
    double *A = (double *)malloc(sizeof(double) * S);
    double *B = (double *)malloc(sizeof(double) * S * D);
    for (long n = 0; n < N; ++n) {
        for (long s = 0; s < S; ++s) A[s] = A0 ? A0[n * S + s] : 0.0;
        for (long i = 0; i < S * D; ++i) B[i] = B0 ? B0[n * S * D + i] : 0.0;
        for (long t = 0; t < T; ++t) {
            const double *k = pk + (n * T + t) * S;
            const double *q = pq + (n * T + t) * S;
            const double *v = V + (n * T + t) * D;
            double *o = out + (n * T + t) * D;
            for (long d = 0; d < D; ++d) o[d] = 0.0;
            for (long s = 0; s < S; ++s) {
                A[s] += k[s];
                double *b = B + s * D;
                for (long d = 0; d < D; ++d) b[d] += k[s] * v[d];
                const double w = q[s] / (A[s] + eps);
                for (long d = 0; d < D; ++d) o[d] += w * b[d];
            }
        }
        if (A_fin) memcpy(A_fin + n * S, A, sizeof(double) * S);
        if (B_fin) memcpy(B_fin + n * S * D, B, sizeof(double) * S * D);
    }
    free(A);
    free(B);
}

/*
 * Exact gradients of oracle_race_fwd for the loss
 *     sum_t dO_t . out_t  +  <gA_in, A_final> + <gB_in, B_final>
 * (gA_in [N,S] / gB_in [N,S,D] may be NULL = 0).  Outputs dpk, dpq [N,T,S],
 * dV [N,T,D] and, when non-NULL, dA0 [N,S], dB0 [N,S,D] (gradient of the
 * carried-in state).  Per (n,s) stream this is race_prefix_mean_flat_bw:
 * pass 1 runs forward over t keeping 1/(A+eps) and
 * alpha_t = -(1/(A+eps))^2 * (pq_t dO_t . B_t); pass 2 runs backward
 * accumulating beta = sum_{t'>=t} pq dO /(A+eps) and alpha_suf, giving
 * dpk = alpha_suf + beta . v_t and the V contribution pk_t * beta.
 */
void oracle_race_bwd(const double *pk, const double *pq, const double *V, const double *dO,
                     long N, long T, long S, long D, double eps,
                     const double *A0, const double *B0,
                     const double *gA_in, const double *gB_in,
                     double *dpk, double *dpq, double *dV,
                     double *dA0, double *dB0)
{
    double *invA = (double *)malloc(sizeof(double) * (T > 0 ? T : 1));
    double *alpha = (double *)malloc(sizeof(double) * (T > 0 ? T : 1));
    double *B = (double *)malloc(sizeof(double) * D);
    double *beta = (double *)malloc(sizeof(double) * D);
    for (long i = 0; i < N * T * D; ++i) dV[i] = 0.0;
    for (long n = 0; n < N; ++n) {
        for (long s = 0; s < S; ++s) {
            double A = A0 ? A0[n * S + s] : 0.0;
            for (long d = 0; d < D; ++d) B[d] = B0 ? B0[(n * S + s) * D + d] : 0.0;
            for (long t = 0; t < T; ++t) {
                const double w = pk[(n * T + t) * S + s];
                const double q = pq[(n * T + t) * S + s];
                const double *v = V + (n * T + t) * D;
                const double *g = dO + (n * T + t) * D;
                A += w;
                double G = 0.0;
                for (long d = 0; d < D; ++d) { B[d] += w * v[d]; G += g[d] * B[d]; }
                const double iA = 1.0 / (A + eps);
                invA[t] = iA;
                alpha[t] = -(iA * iA) * q * G;
                dpq[(n * T + t) * S + s] = G * iA;
            }
            double alpha_suf = gA_in ? gA_in[n * S + s] : 0.0;
            for (long d = 0; d < D; ++d) beta[d] = gB_in ? gB_in[(n * S + s) * D + d] : 0.0;
            for (long t = T - 1; t >= 0; --t) {
                const double w = pk[(n * T + t) * S + s];
                const double q = pq[(n * T + t) * S + s];
                const double *v = V + (n * T + t) * D;
                const double *g = dO + (n * T + t) * D;
                double *gv = dV + (n * T + t) * D;
                alpha_suf += alpha[t];
                double bv = 0.0;
                for (long d = 0; d < D; ++d) {
                    beta[d] += q * g[d] * invA[t];
                    bv += beta[d] * v[d];
                    gv[d] += w * beta[d];
                }
                dpk[(n * T + t) * S + s] = alpha_suf + bv;
            }
            if (dA0) dA0[n * S + s] = alpha_suf;
            if (dB0) for (long d = 0; d < D; ++d) dB0[(n * S + s) * D + d] = beta[d];
        }
    }
    free(invA);
    free(alpha);
    free(B);
    free(beta);
}
