"""Import path of the reference (`from ncaops import nca_ops`, train.py:159,168): the UltraNCA-B200 operator API.
This package only re-exports ultranca_b200.nca_ops so that train.py / benchmark.py drop it in unchanged."""
from ultranca_b200 import nca_ops
from ultranca_b200.nca_ops import step, update_mask

__all__ = ['nca_ops', 'step', 'update_mask']
