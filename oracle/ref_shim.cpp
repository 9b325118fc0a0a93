// C-linkage shim around the reference's own FP32 CPU kernel -- TEST
// INFRASTRUCTURE ONLY (built into oracle/_ref/, which is never committed).
//
// oracle/Makefile compiles this file together with the reference source
// csrc/mla_decode_naive_fp32_cpu.cpp where it lies in the reference checkout,
// so the reference function runs unchanged; this shim only gives it a
// ctypes-friendly unmangled name.  The declaration below restates the
// signature of run_mla_decode_cpu (lechebs/ada-mla csrc/mla_decode.hpp:3-8).

void run_mla_decode_cpu(const float *query, const float *cache, float *out,
                        int num_heads, int head_dim_c, int seq_length);

extern "C" void ref_run_mla_decode_cpu(const float *query, const float *cache,
                                       float *out, int num_heads,
                                       int head_dim_c, int seq_length)
{
    run_mla_decode_cpu(query, cache, out, num_heads, head_dim_c, seq_length);
}
