"""Locate and import the UNMODIFIED reference's PyTorch attention path (TEST INFRASTRUCTURE).

Used by ``tests/golden/make_golden.py`` (to produce the golden fixtures) and by
``bench.py --impl reference`` (to time the reference's own CPU path).  Nothing
in the product package imports it.

Where the reference comes from, in order:
  1. ``VA_REFERENCE_ROOT`` -- a directory holding ``vllm_apple/`` (the source
     tree, or a pip ``--target`` install of it);
  2. ``baseline/_ref`` next to this repository's root (the offline pip install
     of the reference, which travels with the repository to the GPU box).
``reference_source_tree()`` names the reference's SOURCE tree (needed only to
compile its ``kv_write.c``): ``VA_REFERENCE_ROOT``, else the directory that
``baseline/_ref`` was installed from (pip's ``direct_url.json``).

The reference targets an older vLLM layout; ``load_reference_attention`` maps
the names it imports (``vllm.attention.backends.abstract``,
``AttentionMetadataBuilder``/``CommonAttentionMetadata`` in
``vllm.v1.attention.backends.utils``) onto vLLM 0.22 and loads
``vllm_apple/v1/attention/backends/{base_attn,mps_attn}.py`` by path, skipping
the package ``__init__`` files that pull in the Apple worker.  The reference's
own code is executed as is.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import types
from urllib.parse import urlparse

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INSTALLED = os.path.join(REPO, "baseline", "_ref")


def reference_root() -> str | None:
    """Directory holding the reference's ``vllm_apple`` package, or None."""
    env = os.environ.get("VA_REFERENCE_ROOT")
    for cand in ([env] if env else []) + [INSTALLED]:
        if cand and os.path.isfile(os.path.join(cand, "vllm_apple", "v1", "attention",
                                                "backends", "mps_attn.py")):
            return cand
    return None


def reference_source_tree() -> str | None:
    """The reference's source tree (with ``vllm_apple/metal/native/kv_write.c``)."""
    env = os.environ.get("VA_REFERENCE_ROOT")
    cands = [env] if env else []
    if os.path.isdir(INSTALLED):
        for d in os.listdir(INSTALLED):
            p = os.path.join(INSTALLED, d, "direct_url.json")
            if d.startswith("vllm_apple") and d.endswith(".dist-info") and os.path.isfile(p):
                with open(p) as f:
                    url = json.load(f).get("url", "")
                if url.startswith("file://"):
                    cands.append(urlparse(url).path)
    for c in cands:
        if c and os.path.isfile(os.path.join(c, "vllm_apple", "metal", "native", "kv_write.c")):
            return c
    return None


def load_reference_attention(root: str | None = None):
    """Import the reference's ``mps_attn`` module (with ``base_attn``) from ``root``."""
    root = root or reference_root()
    if root is None:
        raise FileNotFoundError("reference not found: set VA_REFERENCE_ROOT or install it "
                                "into baseline/_ref")
    import vllm.v1.attention.backend as vb
    import vllm.v1.attention.backends.utils as vu
    from vllm.utils.torch_utils import is_quantized_kv_cache

    abstract = types.ModuleType("vllm.attention.backends.abstract")
    for n in ("AttentionBackend", "AttentionImpl", "AttentionLayer", "AttentionType"):
        setattr(abstract, n, getattr(vb, n))
    abstract.is_quantized_kv_cache = is_quantized_kv_cache
    sys.modules["vllm.attention.backends.abstract"] = abstract
    for n in ("AttentionMetadataBuilder", "CommonAttentionMetadata"):
        if not hasattr(vu, n):
            setattr(vu, n, getattr(vb, n))
    for name, sub in (("vllm_apple", "vllm_apple"), ("vllm_apple.v1", "vllm_apple/v1"),
                      ("vllm_apple.v1.attention", "vllm_apple/v1/attention"),
                      ("vllm_apple.v1.attention.backends", "vllm_apple/v1/attention/backends")):
        m = types.ModuleType(name)
        m.__path__ = [os.path.join(root, sub)]
        sys.modules[name] = m
    mods = {}
    for stem in ("base_attn", "mps_attn"):
        path = os.path.join(root, "vllm_apple/v1/attention/backends", stem + ".py")
        full = "vllm_apple.v1.attention.backends." + stem
        spec = importlib.util.spec_from_file_location(full, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[full] = mod
        spec.loader.exec_module(mod)
        mods[stem] = mod
    return mods["mps_attn"]
