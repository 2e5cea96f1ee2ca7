// Host entry points over the decode attention's chunk rules
// (hymt2_b200/csrc/hy_attn.cuh: attn_chunk_len, attn_chunk_len_wide,
// attn_max_chunks) for the CPU test of their properties; compiled by
// tests/test_attn_rule.py with nvcc (the header is CUDA source) and run on the
// host only.
#include "../hymt2_b200/csrc/hy_attn.cuh"

extern "C" {
// chunk lengths for positions 0 .. n-1: the persistent kernel's rule into
// len[], the per-layer kernels' rule into wide[]
void ar_rules(int kv_heads, int units, int n, int *len, int *wide) {
    for (int pos = 0; pos < n; pos++) {
        len[pos] = hyk::attn_chunk_len(pos, kv_heads, units);
        wide[pos] = hyk::attn_chunk_len_wide(pos, kv_heads, units);
    }
}
int ar_max_chunks(int ctx) { return hyk::attn_max_chunks(ctx); }
int ar_max_units() { return hyk::kMaxUnits; }
int ar_max_units_wide() { return hyk::kMaxUnitsWide; }
int ar_chunk_max() { return hyk::kChunkMax; }
}
