"""Model weight I/O in the reference's JSON format (src/utils/serialization.ts).

A serialized model is ``{"version", "name", "timestamp", "architecture",
"parameters": [{"name", "shape", "data", "requiresGrad"}], "metadata"}`` with
parameters in ``namedParameters()`` order and ``data`` a flat list of
numbers.  Loading parses the JSON once and copies each parameter straight into
the module's device buffer.  The browser-only helpers keep the reference's
behaviour outside a browser (they raise, or report nothing saved).
"""
from __future__ import annotations

import datetime as _dt
import json
from typing import Dict, Optional, Tuple

import numpy as np

from .layers import Module, _torch

__all__ = [
    "getStateDict", "loadStateDict", "serializeModel", "deserializeModel", "saveModelToJSON",
    "loadModelFromJSON", "getModelSize", "downloadModel", "saveModelToStorage",
    "loadModelFromStorage", "listSavedModels", "deleteSavedModel",
]


def getStateDict(module: Module) -> Dict[str, dict]:
    """serialization.ts:40-52: name -> {"tensor": host copy, "requiresGrad"}."""
    out = {}
    for name, p in module.namedParameters():
        out[name] = {"tensor": p.tensor.detach().cpu().numpy().astype(np.float32).copy(),
                     "requiresGrad": True}
    return out


def loadStateDict(module: Module, stateDict: Dict[str, dict],
                  strict: bool = True) -> Tuple[list, list]:
    """serialization.ts:57-115: copy matching parameters into the module;
    returns (missing, unexpected) and raises on a shape mismatch or, when
    strict, on any missing or unexpected name."""
    torch = _torch()
    named = dict(module.namedParameters())
    missing, unexpected = [], []
    for name in stateDict:
        if name not in named:
            unexpected.append(name)
    for name, p in named.items():
        saved = stateDict.get(name)
        if saved is None:
            missing.append(name)
            continue
        t = saved["tensor"] if isinstance(saved, dict) else saved
        arr = np.asarray(t.cpu().numpy() if hasattr(t, "cpu") else t, dtype=np.float32)
        want = tuple(int(v) for v in p.tensor.shape)
        if tuple(arr.shape) != want:
            if strict:
                raise ValueError(f'Shape mismatch for parameter "{name}": expected '
                                 f'[{",".join(map(str, want))}], got '
                                 f'[{",".join(map(str, arr.shape))}]')
            missing.append(name)
            continue
        src = torch.from_numpy(np.ascontiguousarray(arr))
        if p.tensor.is_cuda:
            p.tensor.copy_(src.to(p.tensor.device, non_blocking=False))
        else:
            p.tensor = src.clone()
    if strict and (missing or unexpected):
        raise ValueError(f"State dict mismatch: missing=[{', '.join(missing)}], "
                         f"unexpected=[{', '.join(unexpected)}]")
    return missing, unexpected


def serializeModel(module: Module, name: str = "model",
                   metadata: Optional[dict] = None) -> dict:
    """serialization.ts:120-156."""
    params = []
    for pname, p in module.namedParameters():
        arr = p.tensor.detach().cpu().numpy().astype(np.float32)
        params.append({"name": pname, "shape": [int(v) for v in arr.shape],
                       "data": [float(v) for v in arr.reshape(-1)], "requiresGrad": True})
    meta = {"numParameters": sum(len(p["data"]) for p in params)}
    meta.update(metadata or {})
    now = _dt.datetime.now(_dt.timezone.utc)
    stamp = now.strftime("%Y-%m-%dT%H:%M:%S.") + f"{now.microsecond // 1000:03d}Z"
    return {"version": "1.0.0", "name": name, "timestamp": stamp,
            "architecture": type(module).__name__, "parameters": params, "metadata": meta}


def deserializeModel(serialized: dict) -> Dict[str, dict]:
    """serialization.ts:161-177: each parameter's data rounded to f32."""
    out = {}
    for p in serialized["parameters"]:
        arr = np.asarray(p["data"], dtype=np.float64).astype(np.float32)
        out[p["name"]] = {"tensor": arr.reshape([int(v) for v in p["shape"]]),
                          "requiresGrad": bool(p.get("requiresGrad", True))}
    return out


def saveModelToJSON(module: Module, name: str = "model", metadata: Optional[dict] = None) -> str:
    """serialization.ts:182-189 (two-space indentation, like JSON.stringify)."""
    return json.dumps(serializeModel(module, name, metadata), indent=2)


def loadModelFromJSON(module: Module, text: str, strict: bool = True) -> dict:
    """serialization.ts:194-204."""
    serialized = json.loads(text)
    missing, unexpected = loadStateDict(module, deserializeModel(serialized), strict)
    return {"model": serialized, "missing": missing, "unexpected": unexpected}


def getModelSize(module: Module) -> dict:
    """serialization.ts:299-325."""
    n = sum(int(p.tensor.numel()) for p in module.parameters())
    b = n * 4
    if b < 1024:
        fmt = f"{b} B"
    elif b < 1024 * 1024:
        fmt = f"{b / 1024:.2f} KB"
    else:
        fmt = f"{b / (1024 * 1024):.2f} MB"
    return {"parameters": n, "bytes": b, "formatted": fmt}


# ---- browser-only helpers (serialization.ts:209-294): no DOM or localStorage here
def downloadModel(module: Module, filename: str = "model.json", metadata=None) -> None:
    raise RuntimeError("downloadModel is only available in browser environment")


def saveModelToStorage(module: Module, key: str, metadata=None) -> None:
    raise RuntimeError("saveModelToStorage is only available in browser environment")


def loadModelFromStorage(module: Module, key: str, strict: bool = True):
    raise RuntimeError("loadModelFromStorage is only available in browser environment")


def listSavedModels() -> list:
    return []


def deleteSavedModel(key: str) -> bool:
    return False
