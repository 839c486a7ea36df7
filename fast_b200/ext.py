"""Imports the in-tree drop-in modules ``fastAgg`` and ``sampler_core``.

They are built into ``fast_b200/_ext`` (``python -m fast_b200.build``).
``install_dropin()`` puts that directory on ``sys.path`` so unmodified
reference code (``import fastAgg``, ``from sampler_core import ParallelSampler``)
picks them up.  A missing build raises ImportError; nothing falls back.
"""
import importlib
import importlib.util
import os
import sys

import torch  # noqa: F401  (the shims link against libtorch; load it first)

EXT_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ext")


def install_dropin():
    if EXT_DIR not in sys.path:
        sys.path.insert(0, EXT_DIR)
    return EXT_DIR


def _load(name):
    path = os.path.join(EXT_DIR, name + ".so")
    if not os.path.exists(path):
        raise ImportError("fast_b200: %s is not built (run `python -m fast_b200.build`)" % path)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules.setdefault(name, mod)
    return mod


fastAgg = _load("fastAgg")
sampler_core = _load("sampler_core")
