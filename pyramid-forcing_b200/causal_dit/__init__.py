"""Random-init causal Wan2.1-T2V-1.3B DiT driving the B200 MegaCache.

The caller of the cache path (``wan/modules/causal_model.py`` and the few-step
block loop of ``pipeline/causal_inference.py:445-502`` in the reference),
rebuilt so the benchmark can time latent frames per second over the whole
DiT: QKV / O / FFN / modulation GEMMs on cuBLAS (torch), the self-attention
through ``MegaCache.update`` / ``attend`` (this library's kernels), query RoPE
through ``pkv_rope_q``, and the cross-attention over the cached 512-token text
K/V through the library's ragged attention kernel.  Text encoder and VAE are
outside (the text context is a given [1, 512, 4096] tensor).
"""
from .model import CausalWanDiT, WanConfig  # noqa: F401
from .pipeline import generate_video  # noqa: F401
