"""State dicts for the CUDA sparse layers and folded stacks.

The reference saves a raw layer as {ptrs, indices, weights, importance,
value_scale, importance_scale} and restores weights and the two scale
vectors only (sili/sparse_rnn.py:817-851): importance, the optimiser state
and the layout's headroom start fresh after a reload.  ``state_dict`` here
keeps those keys (so the reference's own loader accepts the dict) and adds
``image``: the layer's checkpoint image (``sili_layer_save_state``), from
which ``load_state_dict`` restores the whole training state, so training
continues bit for bit.  A dict without ``image`` loads the reference's way.
"""
from __future__ import annotations

import numpy as np


def state_dict(layer) -> dict:
    n = layer.n_inputs
    return {
        "ptrs": np.array(layer.ptrs),
        "indices": np.array(layer.indices),
        "weights": np.array(layer.weights_vals),
        "importance": np.array(layer.importance),
        "value_scale": np.array([layer.get_value_scale(r) for r in range(n)], dtype=np.float32),
        "importance_scale": np.array([layer.get_importance_scale(r) for r in range(n)], dtype=np.float32),
        "image": layer.save_state(),
    }


def load_state_dict(layer, d: dict) -> None:
    if "image" in d:
        layer.load_state(np.ascontiguousarray(d["image"], np.uint8))
        return
    # the reference's restore (sili/sparse_rnn.py:840-851)
    layer.load_weights(np.asarray(d["ptrs"], np.int32), np.asarray(d["indices"], np.int32),
                       np.asarray(d["weights"], np.float32))
    for r in range(layer.n_inputs):
        layer.set_value_scale_raw(r, float(d["value_scale"][r]))
        layer.set_importance_scale_raw(r, float(d["importance_scale"][r]))
