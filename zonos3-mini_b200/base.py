"""The operator API every layer module implements, with the reference's checkpoint semantics
(servers/sgl/src/zonos3_sgl/layers/base.py:16-144): tensors are plain attributes, attributes whose name starts
with ``_`` are caches and never part of a checkpoint, ``state_dict`` / ``load_state_dict`` walk child operators
by attribute name, and a top-level load is strict (leftover keys raise ``RuntimeError``)."""

from __future__ import annotations

import re
from typing import Any

import torch

StateDict = dict[str, torch.Tensor]


def _key(prefix: str, name: str) -> str:
    return f"{prefix}.{name}" if prefix else name


class BaseOP:
    def forward(self, *args: Any, **kwargs: Any) -> Any:  # pragma: no cover - interface
        raise NotImplementedError

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def state_dict(self, *, prefix: str = "", result: StateDict | None = None) -> StateDict:
        result = {} if result is None else result
        for name, value in self.__dict__.items():
            if name.startswith("_"):
                continue
            if isinstance(value, torch.Tensor):
                result[_key(prefix, name)] = value
            elif isinstance(value, BaseOP):
                value.state_dict(prefix=_key(prefix, name), result=result)
        return result

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        for name, value in list(self.__dict__.items()):
            if name.startswith("_"):
                continue
            if isinstance(value, torch.Tensor):
                key = _key(prefix, name)
                if key in state_dict:
                    item = state_dict.pop(key)
                else:
                    # per-expert tensors (experts.<i>.<name>) stack into one [E, ...] tensor
                    pattern = re.compile(re.escape(prefix) + r"\.(\d+)\." + re.escape(name) + "$")
                    found = sorted(((int(m.group(1)), k) for k in state_dict if (m := pattern.match(k))))
                    if not found:
                        raise ValueError(f"No weights found in state_dict for {key}")
                    item = torch.stack([state_dict.pop(k) for _, k in found])
                if tuple(item.shape) != tuple(value.shape):
                    raise ValueError(f"Shape mismatch for {key}: param {tuple(value.shape)} vs item {tuple(item.shape)}")
                if item.dtype != value.dtype:
                    if not (item.is_floating_point() and value.is_floating_point()):
                        raise ValueError(f"Dtype mismatch for {key}: param {value.dtype} vs item {item.dtype}")
                    item = item.to(value.dtype)
                setattr(self, name, item.to(value.device) if value.device.type != "meta" else item)
            elif isinstance(value, BaseOP):
                value.load_state_dict(state_dict, prefix=_key(prefix, name), _internal=True)
        if not _internal and state_dict:
            keys = list(state_dict)
            raise RuntimeError(f"Unexpected keys in state_dict: {len(keys)} keys (first 10: {keys[:10]})")

    def to(self, device=None, dtype=None) -> "BaseOP":
        """Moves every checkpoint tensor (and child operator) in place; fp32-only tensors (``_fp32`` names) keep
        their dtype."""
        keep = getattr(self, "_fp32", ())
        for name, value in list(self.__dict__.items()):
            if name.startswith("_"):
                continue
            if isinstance(value, torch.Tensor):
                setattr(self, name, value.to(device=device, dtype=None if name in keep else dtype))
            elif isinstance(value, BaseOP):
                value.to(device, dtype)
        return self


class OPList(BaseOP):
    def __init__(self, ops: list[BaseOP]):
        self.op_list = ops

    def state_dict(self, *, prefix: str = "", result: StateDict | None = None) -> StateDict:
        result = {} if result is None else result
        for i, op in enumerate(self.op_list):
            op.state_dict(prefix=_key(prefix, str(i)), result=result)
        return result

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        for i, op in enumerate(self.op_list):
            op.load_state_dict(state_dict, prefix=_key(prefix, str(i)), _internal=True)
        if not _internal and state_dict:
            keys = list(state_dict)
            raise RuntimeError(f"Unexpected keys in state_dict: {len(keys)} keys (first 10: {keys[:10]})")

    def to(self, device=None, dtype=None) -> "OPList":
        for op in self.op_list:
            op.to(device, dtype)
        return self


class Weight(BaseOP):
    """A named ``.weight`` holder (the checkpoint's ``<module>.weight`` keys)."""

    def __init__(self, shape, dtype=None):
        self.weight = torch.empty(shape, dtype=dtype)
