"""ebr_b200: the B200 (sm_100a) rebuild of the second-order attention hot path of wwillchen/ebr.

``ebr_b200.fused_attn`` is the drop-in for the reference's ``models.fused_attn``; ``ebr_b200.energy`` is the energy
network and latent-descent caller that drives it; ``ebr_b200.runtime`` holds the data-parallel plumbing.
"""

from ebr_b200.fused_attn import fused_attention, implementation

__all__ = ["fused_attention", "implementation"]
