"""Backward pass of the ETHOS expert layer (filled in with the backward kernels)."""


def layer_backward(ctx, gy):
    raise NotImplementedError("EthosExpertLayer backward kernels are not built yet")
