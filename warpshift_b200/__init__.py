"""warpshift_b200: B200-native in-place model switching (delta decode + apply on sm_100a).

Modules:
  delta    -- DeltaWeights drop-in (encode at prepare, fused decode+apply on switch)
  weights  -- worker-side parameter walk, CPU backups and the TP-agreed loader
  synth    -- synthetic model pairs with the benchmark shapes and SGLang TP sharding
  build    -- nvcc build of the in-tree native library
"""

__version__ = "0.1.0"
