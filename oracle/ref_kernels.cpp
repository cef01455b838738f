// ORACLE — test infrastructure only (see oracle/oracle.c).
//
// Exposes the reference's file-local kernels with C linkage so that the tests can call the
// reference itself on isolated inputs.  The reference source is not copied: it is included
// in place from REF_SRC (set by oracle/Makefile) and compiled with the reference's own
// canonical flags.  Wrapped functions: signed_4bit_b128_gemv (src/llama_engine.cpp:233),
// signed_4bit_b128_fused_swiglu (:362), compute_x_block_sums (:496), rms_norm (:87),
// apply_rope (:120), SignedBlock128Matrix::dequantize_embedding_row (:182), sample_top_p (:784).
#include REF_SRC

extern "C" {

static SignedBlock128Matrix ref_make(uint32_t N, uint32_t K, const uint8_t* nib,
                                     const uint16_t* step, const uint16_t* mn) {
    SignedBlock128Matrix m;
    m.out_dim = N;
    m.in_dim = K;
    m.num_blocks = N * (K / 128);
    m.nibbles = nib;
    m.step_bf16 = step;
    m.min_bf16 = mn;
    return m;
}

void ref_gemv(const uint8_t* nib, const uint16_t* step, const uint16_t* mn, uint32_t N, uint32_t K,
              const float* x, const float* xs, float* y) {
    signed_4bit_b128_gemv(ref_make(N, K, nib, step, mn), x, xs, y);
}

void ref_swiglu(const uint8_t* gn, const uint16_t* gs, const uint16_t* gm, const uint8_t* un,
                const uint16_t* us, const uint16_t* um, uint32_t N, uint32_t K, const float* x,
                const float* xs, float* act) {
    signed_4bit_b128_fused_swiglu(ref_make(N, K, gn, gs, gm), ref_make(N, K, un, us, um), x, xs, act);
}

void ref_block_sums(const float* x, size_t K, float* sums) { compute_x_block_sums(x, K, sums); }

void ref_rms_norm(const float* x, const float* w, float* out, size_t n) { rms_norm(x, w, out, n); }

void ref_apply_rope(float* v, size_t n_heads, size_t head_dim, size_t pos, const float* c,
                    const float* s) {
    apply_rope(v, n_heads, head_dim, pos, c, s);
}

void ref_dequant_row(const uint8_t* nib, const uint16_t* step, const uint16_t* mn, uint32_t N,
                     uint32_t K, size_t row, float* out) {
    ref_make(N, K, nib, step, mn).dequantize_embedding_row(row, out);
}

int32_t ref_sample(float* logits, size_t vocab, float temperature, float top_p) {
    return sample_top_p(logits, vocab, temperature, top_p);
}

}  // extern "C"
