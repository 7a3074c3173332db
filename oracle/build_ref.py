"""Compiles the reference's own CPU path for the attention forward -- TEST AND BASELINE
INFRASTRUCTURE ONLY (the reference arm and the cpu_baseline leg of bench.py).

    python oracle/build_ref.py REFERENCE_DIR        (or FA_REFERENCE_DIR=REFERENCE_DIR)

The reference's CPU path is ``attention_reference`` in its ``fa/reference.py`` (lines 8-18 of
aligoldenhat/flash-attention-from-scratch): fp32 upcast, Q K^T / sqrt(d), causal triu mask,
softmax, @ V, in torch. The function is loaded by file path from the reference checkout
(importing the package ``fa`` there would need its compiled CUDA extension), compiled
unmodified with ``torch.jit.script`` and saved to ``oracle/_ref/attention_reference.pt``: the
archive holds the TorchScript IR of the reference's own code, so it runs the reference's torch
ops without the reference checkout and travels to the GPU box like a built library
(``oracle/_ref/`` is git-ignored). Before the file is written the scripted function is checked
bit for bit against the original on a causal and a non-causal case.
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "attention_reference.pt"


def _stamp() -> Path:
    return OUT.with_name(OUT.name + ".stamp")


def build(reference: Path | None, quiet: bool = False) -> Path | None:
    """Builds OUT from `reference` (a checkout of the reference); returns None when the
    reference's fa/reference.py is not there."""
    if reference is None:
        return None
    src = Path(reference) / "fa" / "reference.py"
    if not src.exists():
        if not quiet:
            print(f"[build_ref] {src} not found; skipped")
        return None
    import torch

    digest = hashlib.sha256(src.read_bytes() + torch.__version__.encode()).hexdigest()
    if OUT.exists() and _stamp().exists() and _stamp().read_text().strip() == digest:
        return OUT
    spec = importlib.util.spec_from_file_location("fa_reference_cpu_path", src)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("ignore", DeprecationWarning)
        scripted = torch.jit.script(mod.attention_reference)
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(1, 2, 70, 64, generator=g).half() for _ in range(3))
    for causal in (False, True):
        want = mod.attention_reference(q, k, v, causal=causal)
        got = scripted(q, k, v, causal)
        if not torch.equal(want, got):
            raise RuntimeError("scripted attention_reference differs from the original")
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".pt.tmp")
    torch.jit.save(scripted, str(tmp))
    os.replace(tmp, OUT)
    _stamp().write_text(digest + "\n")
    if not quiet:
        print(f"[build_ref] {OUT}")
    return OUT


def load():
    """The compiled reference function (q, k, v, causal) -> fp32 O, or None if not built."""
    if not OUT.exists():
        return None
    import warnings

    import torch

    with warnings.catch_warnings():
        warnings.simplefilter("ignore", DeprecationWarning)  # TorchScript is deprecated, still shipped
        return torch.jit.load(str(OUT), map_location="cpu")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FA_REFERENCE_DIR")
    if ref is None:
        raise SystemExit("usage: python oracle/build_ref.py REFERENCE_DIR (or set FA_REFERENCE_DIR)")
    print(build(Path(ref)))
