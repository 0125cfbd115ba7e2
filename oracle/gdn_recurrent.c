/* gdn_recurrent.c -- TEST INFRASTRUCTURE ONLY (the oracle).
 *
 * CPU restatement of the reference's fp32 scalar gated-delta-rule recurrence, the definition
 * of the qwen35moe_gdn_prefill maths:
 *   kernels/qwen35moe_gdn_prefill.cu:31-100  (gdn_ref_kernel)
 *   kernels/qwen35moe_gdn_prefill.py:139-151 (kernel_fn: default scale = D^-0.5)
 *
 * Only tests, the smoke check and the benchmark's CPU-baseline leg call this file.  The product
 * path (the CUDA library) never links or calls it.
 *
 * Per (sequence n, value head h, value column c) the state row S[c][0..dk) evolves token by
 * token exactly in the reference's order:
 *   kh     = h % hk                                   (cu:48, interleaved GQA)
 *   gamma  = exp(g[t,h])                              (cu:66)
 *   kv     = sum_i S[c][i] * k[t,kh,i]                (cu:68-79)
 *   delta  = (v[t,h,c] - gamma * kv) * beta[t,h]      (cu:80)
 *   S[c][i]= gamma * S[c][i] + k[t,kh,i] * delta      (cu:85)
 *   o[t,h,c] = scale * sum_i S[c][i] * q[t,kh,i]      (cu:86-92, with the UPDATED state)
 * and the final S is written out (cu:95-99).  State layout is [v][k] ("[v_col, k_row]").
 *
 * The two dot products are summed the way the reference's warp does it: 32 lane partials
 * (lane l owns elements l, l+32, l+64, ...), then a butterfly over the partials
 * (cu:22-29).  This keeps the fp32 rounding close to the reference's own kernel.
 *
 * Varlen: token ranges per sequence come from cu_seqlens (nseq + 1 entries).  A batch of B
 * equal-length sequences is the special case cu_seqlens = {0, T, 2T, ...}.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define LANES 32

static float lane_tree_sum(float* part) {
  /* butterfly: offsets 16, 8, 4, 2, 1 -- every lane ends with the same value */
  for (int off = LANES / 2; off > 0; off >>= 1) {
    float nxt[LANES];
    for (int l = 0; l < LANES; ++l) nxt[l] = part[l] + part[l ^ off];
    memcpy(part, nxt, sizeof(nxt));
  }
  return part[0];
}

static float dot_lanes(const float* a, const float* b, int n) {
  float part[LANES];
  for (int l = 0; l < LANES; ++l) part[l] = 0.0f;
  for (int r = 0; r < n / LANES; ++r) {
    for (int l = 0; l < LANES; ++l) part[l] += a[r * LANES + l] * b[r * LANES + l];
  }
  for (int i = (n / LANES) * LANES; i < n; ++i) part[i % LANES] += a[i] * b[i];
  return lane_tree_sum(part);
}

/* Returns 0 on success, -1 on bad arguments.
 * q, k      : [total, hk, dk]
 * v, out    : [total, hv, dv]
 * g, beta   : [total, hv]
 * state_in  : [nseq, hv, dv, dk]   (may be NULL: zero initial state)
 * state_out : [nseq, hv, dv, dk]
 */
int oracle_gdn_recurrent(const float* q, const float* k, const float* v, const float* g, const float* beta,
                         const float* state_in, float* out, float* state_out, const int64_t* cu_seqlens, int nseq,
                         int hk, int hv, int dk, int dv, float scale, int nthreads) {
  if (nseq <= 0 || hk <= 0 || hv <= 0 || dk <= 0 || dv <= 0 || (hv % hk) != 0) return -1;
  if (dk % LANES != 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  const long units = (long)nseq * hv;
#pragma omp parallel for schedule(dynamic, 1)
  for (long u = 0; u < units; ++u) {
    const int n = (int)(u / hv);
    const int h = (int)(u % hv);
    const int kh = h % hk;
    const int64_t t0 = cu_seqlens[n], t1 = cu_seqlens[n + 1];
    float* S = state_out + ((size_t)n * hv + h) * (size_t)dv * dk;
    if (state_in) {
      memcpy(S, state_in + ((size_t)n * hv + h) * (size_t)dv * dk, sizeof(float) * (size_t)dv * dk);
    } else {
      memset(S, 0, sizeof(float) * (size_t)dv * dk);
    }
    for (int64_t t = t0; t < t1; ++t) {
      const float* kt = k + ((size_t)t * hk + kh) * dk;
      const float* qt = q + ((size_t)t * hk + kh) * dk;
      const float* vt = v + ((size_t)t * hv + h) * dv;
      const float bt = beta[(size_t)t * hv + h];
      const float gt = expf(g[(size_t)t * hv + h]);
      float* ot = out + ((size_t)t * hv + h) * dv;
      for (int c = 0; c < dv; ++c) {
        float* row = S + (size_t)c * dk;
        const float kv = dot_lanes(row, kt, dk);
        const float delta = (vt[c] - gt * kv) * bt;
        for (int i = 0; i < dk; ++i) row[i] = gt * row[i] + kt[i] * delta;
        ot[c] = dot_lanes(row, qt, dk) * scale;
      }
    }
  }
  return 0;
}
