/*
 * CPU oracle for the MLA decode path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
 * the `--impl reference` arm) may load this library; it is the checker and the
 * reported CPU baseline, never the product path.  The product path
 * (ada-mla_b200/) has no CPU fallback and never links this file.
 *
 * This is a plain-C restatement of the reference's FP32 CPU kernel
 * `run_mla_decode_cpu` (lechebs/ada-mla csrc/mla_decode_naive_fp32_cpu.cpp:5-61):
 *
 *   1. S[i][j] = (sum_k q[i][k] * c[j][k]) / sqrt(head_dim_c)     (cpp:15-26)
 *      -- fp32 accumulation in k order, then one division by the
 *         double-precision sqrt(head_dim_c), rounded back to fp32.
 *   2. row softmax with max subtraction: max over j, sum of exp(S - max),
 *      then P = exp(S - max) / sum                                  (cpp:28-48)
 *      -- the reference's unqualified exp() on a float expression resolves to
 *         the double-precision ::exp, and the fp32 running sum is updated in
 *         double then rounded; restating that makes this file bit-exact with
 *         the reference build (checked by tests/test_oracle.py).
 *   3. out[i][j] = sum_k P[i][k] * c[k][j] for j < head_dim_c, i.e. over ALL
 *      head_dim_c columns (576), not only the 512 latent ones      (cpp:50-58)
 *
 * Its parity is pinned by tests/golden (vectors produced by the reference's own
 * function compiled from its sources by oracle/Makefile) and, where the
 * reference sources are present, directly against oracle/_ref.
 *
 * Callers that want the weight-absorbed decode softmax(scale * Q C^T) C[:, :512]
 * pass Q * (scale * sqrt(head_dim_c)) and keep the first 512 output columns.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Faithful restatement of run_mla_decode_cpu (single-threaded, fp32 state). */
int mla_oracle_decode_f32(const float *query, /* [num_heads, head_dim_c] */
                          const float *cache, /* [seq_length, head_dim_c] */
                          float *out,         /* [num_heads, head_dim_c] */
                          int num_heads, int head_dim_c, int seq_length)
{
    if (num_heads < 0 || head_dim_c <= 0 || seq_length <= 0)
        return -1;
    float *tmp = (float *)malloc(sizeof(float) * (size_t)num_heads * (size_t)seq_length);
    if (!tmp)
        return -2;
    const double inv_den = sqrt((double)head_dim_c);

    for (int i = 0; i < num_heads; ++i) {
        const float *qi = query + (size_t)i * head_dim_c;
        float *ti = tmp + (size_t)i * seq_length;
        for (int j = 0; j < seq_length; ++j) {
            const float *cj = cache + (size_t)j * head_dim_c;
            float acc = 0.0f;
            for (int k = 0; k < head_dim_c; ++k)
                acc += qi[k] * cj[k];
            ti[j] = (float)((double)acc / inv_den);
        }
    }

    for (int i = 0; i < num_heads; ++i) {
        float *ti = tmp + (size_t)i * seq_length;
        float mx = ti[0];
        for (int j = 0; j < seq_length; ++j)
            if (ti[j] > mx)
                mx = ti[j];
        float sum = 0.0f;
        for (int j = 0; j < seq_length; ++j)
            sum = (float)((double)sum + exp((double)(ti[j] - mx)));
        for (int j = 0; j < seq_length; ++j)
            ti[j] = (float)(exp((double)(ti[j] - mx)) / (double)sum);
    }

    for (int i = 0; i < num_heads; ++i) {
        const float *ti = tmp + (size_t)i * seq_length;
        float *oi = out + (size_t)i * head_dim_c;
        for (int j = 0; j < head_dim_c; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < seq_length; ++k)
                acc += ti[k] * cache[(size_t)k * head_dim_c + j];
            oi[j] = acc;
        }
    }
    free(tmp);
    return 0;
}

/*
 * Same algorithm in double precision with an explicit softmax scale and an
 * explicit number of value columns: out = softmax(scale * Q C^T) C[:, :dv].
 * Used by the tests as a high-precision second opinion (it is not a reference
 * function; the fp32 restatement above is the pinned oracle).
 */
int mla_oracle_decode_f64(const float *query, const float *cache, float *out,
                          int num_heads, int head_dim_c, int head_dim_v,
                          int seq_length, double scale)
{
    if (num_heads < 0 || head_dim_c <= 0 || head_dim_v <= 0 || head_dim_v > head_dim_c ||
        seq_length <= 0)
        return -1;
    double *s = (double *)malloc(sizeof(double) * (size_t)seq_length);
    double *o = (double *)malloc(sizeof(double) * (size_t)head_dim_v);
    if (!s || !o) {
        free(s);
        free(o);
        return -2;
    }
    for (int i = 0; i < num_heads; ++i) {
        const float *qi = query + (size_t)i * head_dim_c;
        double mx = -INFINITY;
        for (int j = 0; j < seq_length; ++j) {
            const float *cj = cache + (size_t)j * head_dim_c;
            double acc = 0.0;
            for (int k = 0; k < head_dim_c; ++k)
                acc += (double)qi[k] * (double)cj[k];
            s[j] = acc * scale;
            if (s[j] > mx)
                mx = s[j];
        }
        double sum = 0.0;
        memset(o, 0, sizeof(double) * (size_t)head_dim_v);
        for (int j = 0; j < seq_length; ++j) {
            double p = exp(s[j] - mx);
            sum += p;
            const float *cj = cache + (size_t)j * head_dim_c;
            for (int d = 0; d < head_dim_v; ++d)
                o[d] += p * (double)cj[d];
        }
        float *oi = out + (size_t)i * head_dim_v;
        for (int d = 0; d < head_dim_v; ++d)
            oi[d] = (float)(o[d] / sum);
    }
    free(s);
    free(o);
    return 0;
}
