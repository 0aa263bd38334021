"""Reference checkpoints in and out of models that use EthosExpertLayer.

The reference writes two kinds of checkpoints:

* ``pytorch_model.bin`` -- a plain ``CompressedMoEModel.state_dict()``, loaded
  by ``model.load_state_dict(torch.load(path))`` (notebooks/demo.ipynb, cell 1);
* a DeepSpeed checkpoint directory from ``model_engine.save_checkpoint(dir)``
  (train.py:258-259): a ``latest`` file naming the tag and
  ``<tag>/mp_rank_00_model_states.pt`` whose ``"module"`` entry is the model's
  state_dict (ZeRO-2 keeps full module weights there; optimizer shards live in
  other files and are not needed to run or fine-tune the layer).

``EthosExpertLayer`` has the reference layer's state_dict key for key, so both
load unchanged into a model whose expert layers were swapped
(``swap_expert_layers``), and a model saved with Ethos layers loads back into
the reference.  These helpers only locate, filter and check the entries.
"""

import os

import torch

__all__ = ["load_reference_state_dict", "expert_layer_prefixes", "expert_layer_state", "save_state_dict"]

_LAYER_SUFFIXES = ("expert_latents.weight", "generation_network.net.0.weight", "generation_network.net.2.weight",
                   "router.sub_keys_1.weight", "router.sub_keys_2.weight")


def load_reference_state_dict(path, map_location="cpu"):
    """State dict from a ``pytorch_model.bin``-style file or a DeepSpeed
    checkpoint directory (``latest`` tag, or the only ``global_step*`` /
    tag sub-directory holding ``mp_rank_00_model_states.pt``)."""
    if os.path.isdir(path):
        tag = None
        latest = os.path.join(path, "latest")
        if os.path.isfile(latest):
            with open(latest) as f:
                tag = f.read().strip()
        if tag is None:
            tags = sorted(d for d in os.listdir(path)
                          if os.path.isfile(os.path.join(path, d, "mp_rank_00_model_states.pt")))
            if len(tags) != 1:
                raise FileNotFoundError(f"no unique DeepSpeed tag under {path}: {tags}")
            tag = tags[0]
        f = os.path.join(path, tag, "mp_rank_00_model_states.pt")
        if not os.path.isfile(f):
            f = os.path.join(path, "mp_rank_00_model_states.pt")
        blob = torch.load(f, map_location=map_location, weights_only=False)
        if not isinstance(blob, dict) or "module" not in blob:
            raise ValueError(f"{f} has no 'module' state_dict")
        return blob["module"]
    sd = torch.load(path, map_location=map_location, weights_only=True)
    if isinstance(sd, dict) and "module" in sd and isinstance(sd["module"], dict):
        return sd["module"]
    return sd


def expert_layer_prefixes(state_dict):
    """Prefixes (e.g. ``"layers.3.mlp."``) of every expert layer in a state dict."""
    out = set()
    for k in state_dict:
        if k.endswith(_LAYER_SUFFIXES[0]):
            p = k[: -len(_LAYER_SUFFIXES[0])]
            if all((p + s) in state_dict for s in _LAYER_SUFFIXES):
                out.add(p)
    return sorted(out)


def expert_layer_state(state_dict, prefix):
    """The entries of one expert layer, keys relative to the layer."""
    return {k[len(prefix):]: v for k, v in state_dict.items() if k.startswith(prefix)}


def save_state_dict(model, path):
    """``torch.save(model.state_dict())`` -- the ``pytorch_model.bin`` format the
    reference loads; Ethos layers write the reference's keys."""
    torch.save(model.state_dict(), path)
