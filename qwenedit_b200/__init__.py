"""qwenedit_b200 — B200-native paged prefix K/V cache and fused NVFP4 quantisers for QwenEdit.

Drop-in modules (same API as the reference's):
  qwenedit_b200.paged   <- multi_turn.cache.paged   (PagedKVPool, Match, PoolStats)
  qwenedit_b200.keys    <- multi_turn.cache.keys    (virtual_ids, sequence_ids, root/image/latent keys)
  qwenedit_b200.state   <- multi_turn.state         (dit_pool, encoder_pool, roots, latent LRUs)
  qwenedit_b200.fp4     <- multi_turn.fibo.fp4      (Quantized, norm_scale_fp4, silu_mul_fp4)
  qwenedit_b200.hooks   <- the pool call sites of multi_turn.pipeline.hooks / multi_turn.cache.encoder

All device work runs in libqeb200.so (hand-written sm_100a kernels behind the C ABI in include/qeb200.h).
"""

__version__ = "0.1.0"
