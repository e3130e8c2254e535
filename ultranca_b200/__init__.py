"""UltraNCA-B200: the fused batched NCA step (forward, backward, rollout, update / alive masks, fused optimiser) as
hand-written sm_100a CUDA kernels behind the reference's `impl: cuda` operator API.

    from ultranca_b200 import nca_ops      # step / rollout / update_mask / CHUNK, as ncaops.nca_ops

Submodules load lazily, so `python -m ultranca_b200.build` works before the library exists.
"""
import importlib

__all__ = ['nca_ops', 'step', 'update_mask', 'rollout', 'training', 'sharded']


def __getattr__(name):
    if name in ('nca_ops', 'training', 'sharded'):
        return importlib.import_module(f'.{name}', __name__)
    if name in ('step', 'update_mask', 'rollout'):
        return getattr(importlib.import_module('.nca_ops', __name__), name)
    raise AttributeError(name)
