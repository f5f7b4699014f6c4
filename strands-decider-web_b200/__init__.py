"""s4mm: B200-native (sm_100a) int4 MatMulNBits linear path of the strands-decider-web engine.

Load this directory as a package (its name has hyphens, so import it by path)::

    spec = importlib.util.spec_from_file_location(
        "strands_decider_web_b200", "<dir>/__init__.py", submodule_search_locations=["<dir>"])

Public API: :class:`Context`, :class:`Weight`, :class:`Chain`, :class:`Gemm`, :class:`Manifest`,
:class:`S4Error`, the 24-layer stack runners and the multi-GPU drivers (:mod:`.serve`), and the dispatch-table
tuner (:mod:`.tune`).
"""
from .s4mm import (FAMILY_AUTO, FAMILY_GEMV, FAMILY_TC, LIB_PATH, Chain, Context, Gemm, Manifest, S4Error,  # noqa: F401
                   Weight, WeightCache, cache_prefix, fnv1a32, load_library)


def build(verbose: bool = False) -> str:
    """Compile ``libs4mm.so`` for sm_100a (needs nvcc; no GPU)."""
    from . import builder as _b
    return _b.build(verbose=verbose)
