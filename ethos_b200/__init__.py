"""B200-native ETHOS expert layer: product-key router + reordered hypernetwork
experts, forward and backward, in hand-written sm_100a CUDA behind the
reference's nn.Module interface (see ``ethos_b200.layer``)."""

from .config import EthosConfig, layer_dims
from .decoder import DecoderConfig, EthosDecoder
from .layer import EthosExpertLayer, ExpertGenerationNetwork, ProductKeyRouter, swap_expert_layers

__all__ = ["EthosConfig", "layer_dims", "EthosExpertLayer", "ExpertGenerationNetwork",
           "ProductKeyRouter", "swap_expert_layers", "DecoderConfig", "EthosDecoder"]
