// Builds the reference's own host references for the expert product (TEST INFRASTRUCTURE ONLY).
//
// metal/src/iq_parity.cpp is compiled here unmodified, straight from the StrataMetal tree; its main() is
// renamed so this file can expose the functions the reference's iq parity test judges its kernels
// against: quant_host_block (q8_1, :350-382), row_dot (:275-292) over dot_q2_0 / dot_iq2_s, and
// ref_expert (:386-411).  The Metal launchers it also names are satisfied by ref_stubs.cpp and never run.
#define main strata_iq_parity_main
#include "metal/src/iq_parity.cpp"
#undef main

extern "C" {

void ref_quant_q8_1_block(const float* x, uint8_t* y) { quant_host_block(x, y); }

float ref_row_dot(int type, const uint8_t* row, const uint8_t* col, int n_in, int alt) {
    return row_dot(type, row, col, n_in, alt != 0);
}

// One expert over n_tok q8_1 columns; blob = [gate rows | up rows | down rows].
void ref_expert_q8(int gu_type, int d_type, int n_embd, int n_ff, const uint8_t* blob, size_t blob_bytes,
                   const uint8_t* x_q8, int n_tok, float* y) {
    IqExpert e{gu_type, d_type, n_embd, n_ff};
    std::vector<uint8_t> b(blob, blob + blob_bytes);
    std::vector<uint8_t> x(x_q8, x_q8 + (size_t) n_tok * (size_t) (n_embd / 32) * 36u);
    std::vector<float> out = ref_expert(b, x, e, n_tok);
    std::memcpy(y, out.data(), out.size() * sizeof(float));
}

}
