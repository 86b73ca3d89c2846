"""The Hyena mixer as one opaque custom op (the boundary of mixers.py:807-829,
1404-1423).

Under torch.compile the mixer must be a single opaque node that piecewise
compilation splits around: the metadata-dependent host logic of a step
(speculative slot tables, mixed prefill / decode rows) would otherwise be
traced, graph-break and run eagerly.  `torch.ops.evo2_b200.hyena_mixer(
hidden_states, output, token_ids, layer_name)` mutates `output` with the
layer's forward, resolved by name; its fake implementation does nothing, so
compilation never looks inside.  A mixer built with a `compilation_config`
(vLLM's: `static_forward_context`, `splitting_ops`) registers itself there
under its prefix -- a duplicate name is an error, as in the reference -- and
appends the op to `splitting_ops`; engine-free layers are resolved from this
module's registry (the layer constructed last under a name wins).
"""

import sys
import weakref
from typing import Optional

import torch

HYENA_MIXER_OP = "evo2_b200::hyena_mixer"

_layers = weakref.WeakValueDictionary()


def register_layer(prefix: str, layer, compilation_config=None) -> None:
    if compilation_config is not None:
        ctx = compilation_config.static_forward_context
        if prefix in ctx:
            raise ValueError(f"Duplicate layer name: {prefix}")
        ctx[prefix] = layer
        split = getattr(compilation_config, "splitting_ops", None)
        if split is not None and HYENA_MIXER_OP not in split:
            split.append(HYENA_MIXER_OP)
    _layers[prefix] = layer


def resolve_layer(name: str):
    layer = _layers.get(name)
    if layer is None and "vllm.forward_context" in sys.modules:
        try:
            from vllm.forward_context import get_forward_context

            layer = get_forward_context().no_compile_layers.get(name)
        except Exception:  # no engine step in flight
            layer = None
    if layer is None:
        raise KeyError(f"no Hyena mixer registered as {name!r}")
    return layer


@torch.library.custom_op(HYENA_MIXER_OP, mutates_args=("output",))
def hyena_mixer(hidden_states: torch.Tensor, output: torch.Tensor,
                token_ids: Optional[torch.Tensor], layer_name: str) -> None:
    output.copy_(resolve_layer(layer_name)._forward_impl(hidden_states, token_ids))


@hyena_mixer.register_fake
def _hyena_mixer_fake(hidden_states, output, token_ids, layer_name):
    return None
