"""Load/save of the golden fixtures (npz; bf16 tensors stored as uint16 bit patterns)."""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "int32": torch.int32}


def save(name: str, tensors: dict, meta: dict) -> str:
    arrs = {}
    for k, t in tensors.items():
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            arrs[k] = t.view(torch.int16).numpy()
        else:
            arrs[k] = t.numpy()
        arrs["__dtype__" + k] = np.array(str(t.dtype).replace("torch.", ""))
    for k, v in meta.items():
        arrs["__meta__" + k] = np.array(v)
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrs)
    return path


def load(name: str):
    z = np.load(os.path.join(HERE, name + ".npz"))
    tensors, meta = {}, {}
    for k in z.files:
        if k.startswith("__meta__"):
            v = z[k]
            meta[k[8:]] = v.item() if v.shape == () else v
        elif not k.startswith("__dtype__"):
            dt = str(z["__dtype__" + k])
            a = z[k]
            t = torch.from_numpy(a.copy())
            if dt == "bfloat16":
                t = t.view(torch.bfloat16)
            tensors[k] = t
    return tensors, meta


def names(prefix: str = ""):
    return sorted(f[:-4] for f in os.listdir(HERE) if f.endswith(".npz") and f.startswith(prefix))
