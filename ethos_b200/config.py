"""Layer configuration with the reference's attribute names.

The reference reads its expert-layer hyper-parameters off a plain attribute
object (``train.py:28-65`` ``Config``; ``model.py:183-190`` and
``model.py:273-286`` read ``d_model, num_experts, top_k, num_routing_heads,
d_latent, d_intermediate_hypernet, d_query``).  ``EthosConfig`` carries the
same names and the same defaults (``train.py:33-48``), so either object can be
handed to :class:`ethos_b200.EthosExpertLayer`.
"""

import math

__all__ = ["EthosConfig", "layer_dims"]


class EthosConfig:
    """Attribute bag with the reference defaults (``train.py:33-48``)."""

    def __init__(self, d_model=1024, num_experts=512 ** 2, top_k=16,
                 num_routing_heads=8, d_latent=128, d_intermediate_hypernet=512,
                 d_query=512, **extra):
        self.d_model = d_model
        self.num_experts = num_experts
        self.top_k = top_k
        self.num_routing_heads = num_routing_heads
        self.d_latent = d_latent
        self.d_intermediate_hypernet = d_intermediate_hypernet
        self.d_query = d_query
        for k, v in extra.items():
            setattr(self, k, v)

    def __repr__(self):
        keys = ("d_model", "num_experts", "top_k", "num_routing_heads",
                "d_latent", "d_intermediate_hypernet", "d_query")
        return "EthosConfig(" + ", ".join(f"{k}={getattr(self, k)}" for k in keys) + ")"


def layer_dims(config):
    """Return the expert-layer dimensions as a dict of ints.

    ``num_sub_keys`` is ``sqrt(num_experts)``; the reference asserts that it is
    a perfect square (``model.py:191-192``) and so do we.
    """
    n = int(config.num_experts)
    k_sub = int(math.isqrt(n))
    if k_sub * k_sub != n:
        raise ValueError("num_experts must be a perfect square")
    dq = int(config.d_query)
    if dq % 2:
        raise ValueError("d_query must be even (it is split into two halves)")
    return dict(
        d_model=int(config.d_model), num_experts=n, num_sub_keys=k_sub,
        top_k=int(config.top_k), num_heads=int(config.num_routing_heads),
        d_latent=int(config.d_latent), d_hidden=int(config.d_intermediate_hypernet),
        d_query=dq,
    )
