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
    # MiniMind2-small, 512-token prompt, 512 greedy steps (cache grows to 1024 positions)
    "cfg2-minimind2-small-long": ("minimind2-small", 2, 12, 512, 512, [511, 767, 1022]),
    # MiniMind2, 128-token prompt, 1024 greedy steps
    "cfg3-minimind2": ("minimind2", 3, 13, 128, 1024, [127, 640, 1150]),
}

# BASELINE config 4 rows: MiniMind2 sequences whose prompt lengths span the
# workload's [16, 2048] range; each is run through its prompt and then
# CFG4_STEPS decode steps fed the reference's own tokens.
CFG4 = dict(shape="minimind2", model_seed=4, prompt_lens=[16, 300, 700, 1000, 1400, 1800, 2048, 2040],
            prompt_seed0=400, steps=8)
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


def _cfg4_row(args):
    d, i, plen, pseed, steps = args
    s = SHAPES[CFG4["shape"]]
    prompt = synthetic_prompt(pseed, plen, vocab=s.vocab_size)
    ref = ReferenceModel(d, eps=EPS, theta=THETA)
    st = ref.new_state()
    for tok in prompt[:-1]:
        ref.forward_next_token(st, tok)
    tok = prompt[-1]
    argmax, gaps, tki, tkv, full = [], [], [], [], []
    for j in range(steps + 1):
        nxt, logits = ref.forward_token(st, tok, s.vocab_size)
        argmax.append(nxt)
        srt = np.sort(logits)
        gaps.append(float(srt[-1] - srt[-2]))
        idx = np.argsort(-logits, kind="stable")[:16]
        tki.append(idx.astype(np.int32))
        tkv.append(logits[idx].astype(np.float32))
        if j in (0, steps):
            full.append(logits.copy())
        tok = nxt
    return i, prompt, argmax, gaps, tki, tkv, full


def run_cfg4():
    """Eight config-4 rows: after each prompt, the reference's next token, top-2
    gap and top-16 logits at the prompt's last position and at CFG4_STEPS decode
    steps fed its own tokens; full logits at the first and last of these."""
    from multiprocessing import Pool

    c = CFG4
    s = SHAPES[c["shape"]]
    d = write_runtime_model(CACHE / "cfg4-minimind2", c["shape"], c["model_seed"], eps=EPS, theta=THETA)
    jobs = [(d, i, n, c["prompt_seed0"] + i, c["steps"]) for i, n in enumerate(c["prompt_lens"])]
    with Pool(min(len(jobs), 8)) as pool:
        rows = sorted(pool.map(_cfg4_row, jobs))
    np.savez_compressed(
        HERE / "cfg4-minimind2-rows.npz",
        shape=json.dumps(s.__dict__), model_seed=c["model_seed"], eps=EPS, theta=THETA,
        prompt_lens=np.array(c["prompt_lens"], np.int32), prompt_seeds=np.array([j[3] for j in jobs], np.int32),
        prompts=np.concatenate([np.array(r[1], np.int32) for r in rows]),
        argmax=np.array([r[2] for r in rows], np.int32), top2gap=np.array([r[3] for r in rows], np.float32),
        topk_idx=np.array([r[4] for r in rows], np.int32), topk_val=np.array([r[5] for r in rows], np.float32),
        full_logits=np.array([r[6] for r in rows], np.float32),
    )
    print("cfg4-minimind2-rows:", [r[2] for r in rows])


def toy_cli():
    out = subprocess.run([str(REF_CLI), "--tokens", "1,2", "--max-new-tokens", "4"], capture_output=True, text=True,
                         check=True).stdout
    (HERE / "toy_cli.txt").write_text(out)
    print(out)


if __name__ == "__main__":
    # python tests/golden/make_golden.py [case ...]   (default: every case and the toy CLI answer)
    for name in sys.argv[1:] or list(CASES) + ["cfg4-minimind2-rows"]:
        if name == "cfg4-minimind2-rows":
            run_cfg4()
        else:
            run_case(name, *CASES[name])
    if len(sys.argv) == 1:
        toy_cli()
