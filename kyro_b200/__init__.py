"""kyro_b200 -- the speculative-decoding verify step of Kyro, B200-native.

Host-side mirror of the reference's verify-path interfaces over the C ABI
of include/kyro_spec.h (libkyro_spec.so, sm_100a only):

  PagedAttention          src/model/attention_kernel.rs:4-31
  SpeculativeVerifier     src/speculative.rs:286-339 (verify_drafts)
  DeviceBlockManager      src/scheduler/block_manager.rs:15-153

Lower-level operators live in kyro_b200.verify.  Importing the package does
not need a GPU; calling an operator needs the built library and a B200.
"""
from ._lib import (ACCEPT_GREEDY, ACCEPT_GREEDY_REF, ACCEPT_STOCHASTIC, EXPORTS, KyroError,
                   LIB_PATH)

__version__ = "0.1.0"


def __getattr__(name):
    # operator modules import torch; load them on first use
    if name in ("PagedAttention",):
        from .attention import PagedAttention
        return PagedAttention
    if name in ("SpeculativeVerifier", "DraftStrategy"):
        from . import speculative
        return getattr(speculative, name)
    if name == "DeviceBlockManager":
        from .block_manager import DeviceBlockManager
        return DeviceBlockManager
    if name == "Context":
        from .verify import Context
        return Context
    raise AttributeError(name)
