"""B200 (sm_100a) engine for the parakeet.wgsl FastConformer encoder hot path.

The compute lives in ``libpk_b200.so`` (C ABI: include/pk_b200.h), built from
``csrc/`` by ``build.py``.  This package is the host-side mirror of the
reference's operator layer (``kernels``), encoder graph (``encoder``) and
weight-format contract (``runtime_plan``), plus the seeded random-init
package generator used by tests and the benchmark (``synthetic``).

The directory name contains a dot, so import it through ``load()`` in
``__graft_entry__`` or with ``importlib`` under the module name
``parakeet_wgsl_b200``.
"""
from . import _lib, runtime_plan, stitch, synthetic, windows  # noqa: F401
from ._lib import PkError  # noqa: F401

__all__ = ["_lib", "runtime_plan", "stitch", "synthetic", "windows", "PkError", "kernels", "encoder", "engine"]


def __getattr__(name):
    if name in ("kernels", "encoder", "engine"):
        import importlib

        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
