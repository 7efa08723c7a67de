"""B200-native (sm_100a) drop-in for the reversible-Transformer hot path of
LokeshJatangi/Reversability (`src/reversibility`).

Module layout mirrors the reference package (`model`, `reversible`,
`optimized`, `optimized_v3`, `kernels`, `kernels_v3`); the compute runs in
librevk.so (CUDA kernels for sm_100a) through a C ABI, with no CPU fallback.
"""
