"""Regenerate the golden fixtures in tests/golden/ from the REFERENCE itself.

Runs the reference's own fp32 CPU decode path (its unmodified sources compiled
by oracle/build_ref.sh into oracle/_ref/) on seeded synthetic models and
records what it produced. Needs the reference sources on this machine; the
committed .npz files are what the tests use everywhere else.

    python tests/golden/make_golden.py [case ...]
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model  # noqa: E402
from oracle.oracle import REF_CLI, ReferenceModel  # noqa: E402

CACHE = Path("/tmp/mmc_golden_models")

# name: (shape, model seed, prompt seed, prompt length, new tokens, full-logit steps (None = all))
CASES = {
    "tiny": ("tiny", 1, 7, 12, 20, None),
    "tiny-hd64": ("tiny-hd64", 3, 8, 40, 12, None),
    "tiny-hd96-page-cross": ("tiny-hd96", 2, 9, 70, 10, [0, 63, 64, 65, 79]),
    "cfg1-minimind2-small": ("minimind2-small", 1, 5, 5, 16, [4, 19]),
    "tiny-moe": ("tiny-moe", 4, 11, 30, 12, None),
}
EPS, THETA = 1e-5, 1e6


def run_case(name, shape, mseed, pseed, plen, new, full_steps):
    s = SHAPES[shape]
    d = write_runtime_model(CACHE / name, shape, mseed, eps=EPS, theta=THETA)
    prompt = synthetic_prompt(pseed, plen, vocab=s.vocab_size)
    ref = ReferenceModel(d, eps=EPS, theta=THETA)
    st = ref.new_state()
    fed, argmax, top2gap, topk_idx, topk_val, full = [], [], [], [], [], {}
    nxt = None
    generated = []
    for i in range(plen + new - 1):
        tok = prompt[i] if i < plen else nxt
        if i >= plen - 1 and nxt is not None and i >= plen:
            pass
        fed.append(tok)
        nxt, logits = ref.forward_token(st, tok, s.vocab_size)
        if i >= plen - 1:
            generated.append(nxt)
        argmax.append(nxt)
        srt = np.sort(logits)
        top2gap.append(float(srt[-1] - srt[-2]))
        idx = np.argsort(-logits, kind="stable")[:16]
        topk_idx.append(idx.astype(np.int32))
        topk_val.append(logits[idx].astype(np.float32))
        if full_steps is None or i in full_steps:
            full[i] = logits.copy()
    # free-running greedy output through the reference's own generate()
    gen = ReferenceModel(d, eps=EPS, theta=THETA).generate(prompt, new)
    assert gen == generated[: len(gen)], (gen, generated)
    steps = sorted(full)
    np.savez_compressed(
        HERE / f"{name}.npz",
        shape=json.dumps(s.__dict__), model_seed=mseed, eps=EPS, theta=THETA,
        prompt=np.array(prompt, np.int32), fed=np.array(fed, np.int32), argmax=np.array(argmax, np.int32),
        generated=np.array(gen, np.int32), top2gap=np.array(top2gap, np.float32),
        topk_idx=np.stack(topk_idx), topk_val=np.stack(topk_val),
        full_steps=np.array(steps, np.int32), full_logits=np.stack([full[i] for i in steps]).astype(np.float32),
    )
    print(f"{name}: generated {gen}")


def toy_cli():
    out = subprocess.run([str(REF_CLI), "--tokens", "1,2", "--max-new-tokens", "4"], capture_output=True, text=True,
                         check=True).stdout
    (HERE / "toy_cli.txt").write_text(out)
    print(out)


if __name__ == "__main__":
    # python tests/golden/make_golden.py [case ...]   (default: every case and the toy CLI answer)
    for name in sys.argv[1:] or list(CASES):
        run_case(name, *CASES[name])
    if len(sys.argv) == 1:
        toy_cli()
