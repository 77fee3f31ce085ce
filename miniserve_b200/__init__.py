"""B200-native token sampling for miniserve (sm_100a CUDA behind a C ABI).

    from miniserve_b200 import Sampler
    tok = Sampler().sample(logits, temperature=0.7, top_k=50, top_p=0.9, seed=1)
    tokens, probs, status = Sampler().sample_batch(logits_bxv, temperature=T, top_k=K, top_p=P,
                                                   uniforms=U)
"""
from .sampler import Sampler, uniform_for_seed  # noqa: F401

__version__ = "0.1.0"
