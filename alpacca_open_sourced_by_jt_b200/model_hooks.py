"""Install the B200 attention path on an alpaccaroo `Model` instance.

`install(model)` rebinds the methods the engine's forward passes call
(alpaccaroo/model.py:1429-1440 decode, 1331-1341 prefill chunk) to B200
versions with the same signatures:

  _attention_np(q, K, V, group, inv_sqrt)                   model.py:1231
  _attention_batch_np(q, K, V, positions, group, inv_sqrt)  model.py:1254
  _attention_batch_window_np(..., window, kv_start)          model.py:1567
  _rope_np(vec, n_heads, pos)                                model.py:1191
  _rope_batch_np(vecs, n_heads, positions)                   model.py:1211

They read the model's own hyperparameters and its f32 cos/sin tables
(model.py:871-875), so rotations are bit-identical and attention matches to
the tolerances of `kernels.attention_decode` / `cuda.attention_batch`.
A prefill shape no kernel serves (head_dim not a multiple of 4, or above
256) is declined as the reference's GPU tier declines it (cuda.py:1219-1222),
and the model's own class method answers.  Nothing else in the model
changes; `uninstall(model)` restores the class methods.
"""
from __future__ import annotations

import types

import numpy as np
import torch

from . import cuda as _cuda
from . import device as _dev
from . import kernels as _kernels
from ._hostio import to_device, to_host

_HOOKED = ("_attention_np", "_attention_batch_np", "_attention_batch_window_np", "_rope_np",
           "_rope_batch_np")


def _attention_np(self, q, K, V, group: int, inv_sqrt: float):
    hp = self.hp
    return _kernels.attention_decode(q, K, V, group, inv_sqrt).reshape(hp.n_head, hp.head_dim)


def _attention_batch_np(self, q, K, V, positions, group: int, inv_sqrt: float):
    out = _cuda.attention_batch(q, K, V, positions, group, inv_sqrt)
    if out is None:
        # cuda.attention_batch declined the shape (head_dim not a multiple of 4
        # or above 256), exactly as the reference's GPU tier declines: the
        # model keeps its own, unhooked method (model.py:1254-1272)
        return type(self)._attention_batch_np(self, q, K, V, positions, group, inv_sqrt)
    return out


def _attention_batch_window_np(self, q, K, V, positions, group: int, inv_sqrt: float,
                               window: int = 0, kv_start: int = 0):
    out = _cuda.attention_batch(q, K, V, positions, group, inv_sqrt, window, kv_start)
    if out is None:
        # declined shape: the model's own method (model.py:1567-1592)
        return type(self)._attention_batch_window_np(self, q, K, V, positions, group, inv_sqrt,
                                                     window, kv_start)
    return out


def _rope_np(self, vec, n_heads: int, pos: int):
    hp = self.hp
    return _kernels.rope_decode(vec, self._rope_cos[pos], self._rope_sin[pos], n_heads,
                                hp.head_dim, hp.n_rot, hp.rope_style)


def _rope_batch_np(self, vecs, n_heads: int, positions):
    hp = self.hp
    vecs = np.ascontiguousarray(vecs, dtype=np.float32)
    n = len(vecs)
    qd = to_device(vecs.reshape(n, n_heads, hp.head_dim))
    pd = to_device(np.ascontiguousarray(positions, dtype=np.int32))
    cos = _table(self, "_rope_cos")
    sin = _table(self, "_rope_sin")
    _dev.rope_append(qd, None, None, pd, cos, sin, n_rot=hp.n_rot, style=hp.rope_style)
    return to_host(qd).reshape(n, -1)


def _table(self, name):
    """Device copy of the model's f32 rope table, cached on the instance."""
    cache = self.__dict__.setdefault("_b2a_tables", {})
    host = getattr(self, name)
    key = (name, id(host), host.shape)
    t = cache.get(key)
    if t is None:
        t = to_device(np.ascontiguousarray(host, dtype=np.float32))
        if len(cache) > 4:
            cache.clear()
        cache[key] = t
    return t


def install(model) -> None:
    """Route `model`'s attention and RoPE through the B200 kernels."""
    if not torch.cuda.is_available():
        raise RuntimeError("the B200 attention path needs a CUDA device")
    g = globals()
    for name in _HOOKED:
        setattr(model, name, types.MethodType(g[name], model))
    model._b2a_installed = True


def uninstall(model) -> None:
    for name in _HOOKED:
        model.__dict__.pop(name, None)
    model.__dict__.pop("_b2a_tables", None)
    model._b2a_installed = False
