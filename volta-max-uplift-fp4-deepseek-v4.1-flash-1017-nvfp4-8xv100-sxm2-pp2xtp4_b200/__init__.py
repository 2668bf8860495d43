"""B200-native (sm_100a) routed-expert MoE layer: the drop-in for the reference
build's routed-expert FusedMoE quant-method plugin.

Import name: ``b200moe`` (see ``__graft_entry__.load_package``).  Modules:
``moe`` (the plugin: B200NativeMoe, B200NativeMoEMethod), ``packing`` (device
packing and the reference route plan), ``tiers`` (tier map -> slot maps,
expert-parallel placement), ``ep`` (expert-parallel dispatch / combine),
``_lib`` (ctypes binding of libb200moe.so), ``build`` (nvcc build).
"""

from . import _lib, tiers  # noqa: F401

__all__ = ["_lib", "tiers"]
