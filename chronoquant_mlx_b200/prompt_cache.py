"""Save and restore a model's ChronoQuant caches (one per layer) to a file.

The reference has no file format of its own: its caches follow mlx_lm's
prompt-cache protocol (``state`` / ``meta_state``, cache.py:220-263), which
mlx_lm's ``save_prompt_cache`` / ``load_prompt_cache`` write as one
safetensors file.  This module keeps that file layout with torch tensors:

* tensors ``"{i}.{j}"``: array j of layer i's ``state`` -- the reference layout
  (anchors fp16 [B, H, n_kf, D], packed codes uint32 [B, H, n_pf, D/8], scales
  fp16 [B, H, n_pf]), so a file holds exactly what the reference's state holds;
* metadata ``"0.{i}"`` (or ``"0.{i}.{k}"`` for a tuple): layer i's
  ``meta_state`` -- here the cache configuration (strides, bits, dead zones,
  per-layer V bits, layer index, page size), so the file restores
  self-described; ``"1.{key}"``: caller metadata; ``"2.{i}"``: class names.

Restoring imports the arrays into freshly allocated paged storage on the
target device (``cq_import_state``); there is no host compute path.
"""

from __future__ import annotations

import torch

from .cache import ChronoQuantCache

_CLASSES = {"ChronoQuantCache": ChronoQuantCache}


def save_prompt_cache(file_name: str, cache: list, metadata: dict | None = None) -> None:
    """Write the caches' states, meta states, class names and ``metadata``
    (str -> str) to ``file_name`` (safetensors)."""
    from safetensors.torch import save_file
    tensors, meta = {}, {}
    for i, c in enumerate(cache):
        for j, a in enumerate(c.state):
            tensors[f"{i}.{j}"] = a.detach().contiguous().cpu()
        ms = c.meta_state
        if isinstance(ms, str):
            meta[f"0.{i}"] = ms
        else:
            for k, v in enumerate(ms):
                meta[f"0.{i}.{k}"] = str(v)
        meta[f"2.{i}"] = type(c).__name__
    for k, v in (metadata or {}).items():
        meta[f"1.{k}"] = str(v)
    save_file(tensors, file_name, metadata=meta)


def load_prompt_cache(file_name: str, return_metadata: bool = False, device="cuda"):
    """Rebuild the caches saved by ``save_prompt_cache`` on ``device``.
    Returns the list of caches (and the caller metadata if asked)."""
    from safetensors import safe_open
    from safetensors.torch import load_file
    tensors = load_file(file_name)
    with safe_open(file_name, "pt") as f:
        meta = f.metadata() or {}
    n = len([k for k in meta if k.startswith("2.")])
    caches = []
    for i in range(n):
        cls = _CLASSES.get(meta[f"2.{i}"])
        if cls is None:
            raise ValueError(f"unknown cache class {meta[f'2.{i}']!r} in {file_name}")
        c = cls()
        if f"0.{i}" in meta:
            c.meta_state = meta[f"0.{i}"]
        else:
            ks = sorted((int(k.split(".")[2]), v) for k, v in meta.items() if k.startswith(f"0.{i}."))
            c.meta_state = tuple(v for _, v in ks)
        arrays = []
        j = 0
        while f"{i}.{j}" in tensors:
            arrays.append(tensors[f"{i}.{j}"].to(device))
            j += 1
        if arrays:
            c.state = arrays
        caches.append(c)
    if return_metadata:
        return caches, {k[2:]: v for k, v in meta.items() if k.startswith("1.")}
    return caches
