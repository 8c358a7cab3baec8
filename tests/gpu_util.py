"""Helpers shared by the GPU tests: bf16 bit patterns <-> CUDA tensors."""
import numpy as np
import torch


def to_dev_bf16(bits: np.ndarray, device="cuda:0") -> torch.Tensor:
    b = np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)
    return torch.from_numpy(b.copy()).to(device).view(torch.bfloat16)


def from_dev_bf16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_dev(a: np.ndarray, device="cuda:0") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).copy()).to(device)


def bf16_ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 units of last place (sign-magnitude ordering)."""
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)
    return np.abs(key(a_bits) - key(b_bits))


_FRESH_PROFILE = r'''
import importlib, json, sys
import torch
from torch.profiler import ProfilerActivity, profile
from c_gpt2_b200 import ops
ops.init(0)
module, builder, specs = sys.argv[1], sys.argv[2], json.loads(sys.argv[3])
build = getattr(importlib.import_module("tests." + module), builder)
out = []
for spec in specs:
    call = build(*spec)
    call()  # first-call set-up (module loading, symbol lookups) outside the record
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        status = call()
        torch.cuda.synchronize()
    out.append({"status": status,
                "names": [e.name for e in prof.events() if e.device_type.name == "CUDA"]})
print(json.dumps(out))
'''


def kernel_names_fresh(module: str, builder: str, specs: list) -> list[dict]:
    """The CUDA kernels of one call per spec, read back with torch.profiler in
    a fresh Python process: after many profiler sessions one test process can
    reach a state where a session returns no activity records at all.
    tests.<module>.<builder>(*spec) builds the operands on cuda:0 and returns
    the call (whose return value is reported as "status"); the call runs once
    before the recorded one."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "-c", _FRESH_PROFILE, module, builder, json.dumps(specs)],
                       cwd=root, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])
