"""The reference's import name, ``wbridge``, served by ``weightbridge_b200``.

Code written against the reference (``from wbridge import WeightSender, WeightReceiver, ...``,
``wbridge/__init__.py:3-17``; ``from wbridge.frontend import ...``, ``wbridge/frontend/__init__.py:3-6``;
``from wbridge.utils.data import WeightData``; ``wbridge.utils.megatron_utils.convert_to_wb`` and
``wbridge.utils.sglang_utils.convert_to_wb``) runs unchanged on this library.  The submodule
names are registered as aliases of the modules that implement them here; nothing is copied.
"""
import importlib
import sys
import types

from weightbridge_b200 import (WeightData, WeightReceiver, WeightReceiverController, WeightSender,
                               dtype_str_to_torch, dtype_to_str)

__all__ = ["WeightReceiver", "WeightSender", "WeightData", "WeightReceiverController", "dtype_str_to_torch",
           "dtype_to_str"]

# submodule name -> module of this library that provides the same names
_ALIASES = {
    "frontend": "weightbridge_b200.frontend",
    "utils.megatron_utils": "weightbridge_b200.parallel.megatron",
    "utils.sglang_utils": "weightbridge_b200.parallel.sglang",
    "utils.distributed": "weightbridge_b200.control.session",
}


def _install() -> None:
    utils = types.ModuleType(__name__ + ".utils")
    utils.__path__ = []                     # a package, so "wbridge.utils.data" resolves below
    sys.modules[utils.__name__] = utils
    globals()["utils"] = utils
    for sub, target in _ALIASES.items():
        mod = importlib.import_module(target)
        sys.modules[f"{__name__}.{sub}"] = mod
        parent, _, leaf = sub.rpartition(".")
        setattr(utils if parent == "utils" else sys.modules[__name__], leaf, mod)
    # the reference's utils/data.py holds the shard algebra, the dtype helpers and the pair-form
    # alignment check (``_check_shard_compatibility``): one namespace over this library's modules
    shard = importlib.import_module("weightbridge_b200.core.shard")
    data = types.ModuleType(__name__ + ".utils.data")
    data.__dict__.update({k: v for k, v in vars(shard).items() if not k.startswith("__")})
    data.dtype_str_to_torch, data.dtype_to_str = dtype_str_to_torch, dtype_to_str
    data._check_shard_compatibility = shard.check_shard_compatibility
    sys.modules[data.__name__] = data
    utils.data = data


_install()
