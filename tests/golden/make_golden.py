"""Generates the golden attention vectors in tests/golden/ from the REFERENCE's own oracle.

    python tests/golden/make_golden.py REFERENCE_DIR     (a checkout of the reference)

Loads ``attention_reference`` from the reference checkout's fa/reference.py by file path
(importing the package ``fa`` there would need its compiled extension) and runs it on torch
CPU on seeded inputs from fa.synthetic.make_qkv. Writes one .npz per case (q, k, v as fp16;
out as fp32) and cases.json. Run once where the reference is available; the outputs are
committed so the tests never need the reference itself.
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "flash-attention-from-scratch_b200"))

from fa.synthetic import make_qkv  # noqa: E402

CASES = [
    # name, b, h, n, d, causal, seed, scale, outliers
    # cfg0 (the CPU anchor) stores both the non-causal and the causal output ("out_causal").
    ("cfg0", 1, 4, 512, 64, False, 0, 1.0, False),
    ("n1_d64", 1, 2, 1, 64, False, 11, 1.0, False),
    ("n1_d128_causal", 1, 2, 1, 128, True, 12, 1.0, False),
    ("n17_d64_causal", 1, 2, 17, 64, True, 13, 1.0, False),
    ("n65_d128", 1, 2, 65, 128, False, 14, 1.0, False),
    ("n130_d64_causal", 1, 2, 130, 64, True, 15, 1.0, False),
    ("n257_d128_causal", 1, 1, 257, 128, True, 16, 1.0, False),
    ("n300_d64_outliers", 1, 2, 300, 64, False, 4, 1.0, True),
    ("n300_d128_outliers_causal", 1, 1, 300, 128, True, 4, 1.0, True),
    ("large_logits_causal", 1, 2, 256, 64, True, 2, 4.0, False),
]


def main() -> None:
    if len(sys.argv) < 2:
        raise SystemExit("usage: python tests/golden/make_golden.py REFERENCE_DIR")
    ref_root = Path(sys.argv[1])
    spec = importlib.util.spec_from_file_location("fa_reference_oracle", ref_root / "fa" / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    meta = []
    for name, b, h, n, d, causal, seed, scale, outliers in CASES:
        q, k, v = make_qkv(b, h, n, d, seed, scale=scale, outliers=outliers)
        with torch.no_grad():
            out = mod.attention_reference(q, k, v, causal=causal)
            extra = {}
            if name == "cfg0":
                extra["out_causal"] = mod.attention_reference(q, k, v, causal=True).numpy().astype(np.float32)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q=q.numpy(),
            k=k.numpy(),
            v=v.numpy(),
            out=out.numpy().astype(np.float32),
            **extra,
        )
        meta.append(
            dict(
                name=name, b=b, h=h, n=n, d=d, causal=causal, seed=seed, scale=scale, outliers=outliers,
                out_sum=float(out.double().sum()), out_abs_mean=float(out.abs().double().mean()),
                out_abs_max=float(out.abs().max()),
                q_sum=float(q.double().sum()), k_sum=float(k.double().sum()), v_sum=float(v.double().sum()),
            )
        )
        print(name, meta[-1]["out_sum"], meta[-1]["out_abs_mean"])
    (HERE / "cases.json").write_text(json.dumps({"generator": "reference fa/reference.py attention_reference, torch CPU", "torch": torch.__version__, "cases": meta}, indent=1))


if __name__ == "__main__":
    main()
