"""`ncaops.nca_ops` of the reference, served by ultranca_b200.nca_ops (same functions, same module globals)."""
import sys

from ultranca_b200 import nca_ops as _impl

sys.modules[__name__] = _impl  # `nca_ops.CHUNK = ...` and friends act on the one implementation module
