"""Import-path alias: ``mu_space`` is the B200 build in ``muspace_b200``.

Code written against the reference package (``from mu_space.ops import
multi_scale_deformable_attn``, ``from mu_space.patcher import default_patcher``,
``import mu_space.runtime.native``) runs unchanged: every ``mu_space.<sub>``
module listed below is the very same module object as ``muspace_b200.<sub>``,
so monkeypatching one patches the other.
"""

import importlib
import sys

import muspace_b200
from muspace_b200 import *  # noqa: F401,F403
from muspace_b200 import __all__, __version__  # noqa: F401

_SUBMODULES = (
    "ops",
    "ops.multi_scale_deformable_attn",
    "ops.sca_scatter",
    "ops.deformable_aggregation",
    "ops.flash_sca",
    "runtime",
    "runtime.kernel_dispatch",
    "runtime.native",
    "patcher",
    "patcher.runtime",
)
# the reference's module names that differ from this build's
_RENAMED = {"ops.flashbev": "ops.flash_sca"}
for _name in _SUBMODULES:
    sys.modules[f"{__name__}.{_name}"] = importlib.import_module(f"muspace_b200.{_name}")
for _name, _target in _RENAMED.items():
    _module = importlib.import_module(f"muspace_b200.{_target}")
    sys.modules[f"{__name__}.{_name}"] = _module
    _parent, _, _leaf = _name.rpartition(".")
    setattr(sys.modules[f"{__name__}.{_parent}"], _leaf, _module)
ops = muspace_b200.ops
runtime = muspace_b200.runtime
patcher = importlib.import_module("muspace_b200.patcher")
