"""Q38RT B200: a B200-native (sm_100a) decode runtime for GGML K-quant hybrid
Qwen-style models, drop-in behind the Q38RT C ABI (include/q38rt.h).

Submodules:
  build    -- compiles csrc/ into lib/libq38rt_b200.so (nvcc, sm_100a only)
  runtime  -- ctypes binding of the C ABI
  synth    -- seeded synthetic K-quant tensors and activations
"""
