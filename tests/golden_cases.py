"""Loader for the golden fixtures produced by ``tests/golden/make_golden.py``."""

import glob
import os
from typing import Dict, List

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names() -> List[str]:
    names = [os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))]
    return sorted(n for n in names if n != "freqs")


def load_case(name: str) -> Dict[str, object]:
    raw = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    case: Dict[str, object] = {}
    for key in raw.files:
        arr = raw[key]
        if key == "dtype":
            case[key] = torch.float64 if str(arr) == "f64" else torch.float32
        elif key == "flags":
            case[key] = (bool(arr[0]), bool(arr[1]))
        elif arr.size == 0:
            case[key] = None
        else:
            case[key] = torch.from_numpy(arr.copy())
    return case


def load_freqs() -> Dict[int, torch.Tensor]:
    raw = np.load(os.path.join(GOLDEN, "freqs.npz"))
    return {int(k.split("_")[1]): torch.from_numpy(raw[k].copy()) for k in raw.files}
