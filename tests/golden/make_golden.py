"""Generates tests/golden/attention_bmm.npz from the reference's own ``attention_bmm`` (attention.py:15-43).

Runs only where the reference checkout is present: the environment variable REF_DIR names its directory. The
reference package imports
ComfyUI and a HIP loader at module level, which do not exist here, so this script loads ``attention.py`` alone as a
submodule of a bare package object and stubs exactly the two names it imports: ``comfy.ldm.modules.attention
.attention_pytorch`` (only reached with a mask) and the sibling ``hip_attention`` module (only reached by
``attention_hip``). ``attention_bmm`` itself is the reference's unmodified torch code, run on CPU in fp16.
"""
import importlib
import os
import sys
import types

import numpy as np
import torch

REF_DIR = os.environ.get("REF_DIR", "")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "attention_bmm.npz")


def load_reference_attention():
    for name in ("comfy", "comfy.ldm", "comfy.ldm.modules"):
        sys.modules.setdefault(name, types.ModuleType(name))
    stub = types.ModuleType("comfy.ldm.modules.attention")
    stub.attention_pytorch = None
    sys.modules["comfy.ldm.modules.attention"] = stub
    pkg = types.ModuleType("rdna2_reference")
    pkg.__path__ = [REF_DIR]
    sys.modules["rdna2_reference"] = pkg
    sys.modules["rdna2_reference.hip_attention"] = types.ModuleType("rdna2_reference.hip_attention")
    return importlib.import_module("rdna2_reference.attention")


def main():
    if not REF_DIR or not os.path.isfile(os.path.join(REF_DIR, "attention.py")):
        sys.exit("set REF_DIR to the reference checkout (the directory holding attention.py)")
    ref = load_reference_attention()
    g = torch.Generator().manual_seed(20261201)
    cases = {}
    # (B, H, Lq, Lk) in the (B, H, L, D) layout, and one (B, L, H*D) call.
    for name, (b, h, lq, lk) in {"self": (1, 2, 40, 40), "cross": (2, 1, 33, 50)}.items():
        q = torch.randn((b, h, lq, 128), generator=g).half()
        k = torch.randn((b, h, lk, 128), generator=g).half()
        v = torch.randn((b, h, lk, 128), generator=g).half()
        out = ref.attention_bmm(q, k, v, h, skip_reshape=True, skip_output_reshape=True)
        cases.update({f"{name}_q": q.numpy(), f"{name}_k": k.numpy(), f"{name}_v": v.numpy(), f"{name}_out": out.numpy()})
    q = torch.randn((1, 24, 256), generator=g).half()
    k = torch.randn((1, 24, 256), generator=g).half()
    v = torch.randn((1, 24, 256), generator=g).half()
    out = ref.attention_bmm(q, k, v, 2)
    cases.update({"flat_q": q.numpy(), "flat_k": k.numpy(), "flat_v": v.numpy(), "flat_out": out.numpy()})
    np.savez_compressed(OUT, **cases)
    print(OUT, {k: v.shape for k, v in cases.items()})


if __name__ == "__main__":
    main()
