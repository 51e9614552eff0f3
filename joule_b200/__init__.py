"""joule_b200 — B200-native (sm_100a) MoE decode hot path for Joule's Q4 store.

One MoE FFN layer at decode: router softmax/top-k, token-to-expert dispatch,
grouped per-expert gate/up, SwiGLU, down over the Q4 expert store and the
weighted combine, as hand-written CUDA behind a plain C ABI
(include/joule_moe.h, libjoule_moe.so).

  joule_b200.native    library loader (get_dll) and ctypes signatures
  joule_b200.moe       MoELayers (device store + forward), layer_ffn_batch drop-in
  joule_b200.backend   KernelBackend / CudaBackend (q4_gemv, q4_gemm)
  joule_b200.kernel    module-level q4_gemv / q4_gemm
  joule_b200.q4_store  the reference's on-disk Q4 store -> device store
  joule_b200.synth     seeded synthetic inputs for the benchmark shapes
  joule_b200.build     in-tree nvcc build of libjoule_moe.so
"""
__version__ = "0.1.0"
