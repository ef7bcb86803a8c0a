"""Config-3 greedy decode of the full random-init Qwen3.5-4B against the
reference's own decode step and kernels.

The checker, ``oracle.ref_engine.ReferenceKernelEngine``, replays
``QwenEngineFP8Opt.forward``'s default single-token branch (main.py:1509-1604)
with the reference's CUDA kernels (fused_kernels.cu built unmodified into
oracle/_ref).  All engines get the same seeded weights and the same seeded
128-token prompt (ids uniform in [0, 248320)), then 300 greedy steps.

The random-init 4B network amplifies every rounding difference: the oracle's
exact-dequant restatement (``oracle.model.OracleModel``, same arithmetic up to
FP32 summation order) is itself ~3e-2 (rel-l2) away from the reference's
kernels in its logits and flips ~1 greedy token in 15 on near-ties.  So the
bar is that noise floor, measured in the same run: our step kernel must be as
close to the reference as the oracle is (within LOGIT_FLOOR_X of it).

Teacher-forced run: every step feeds the reference's token to all engines, so
one near-tie cannot derail the rest of the run.  Per step
  * our fused argmax is the first-index argmax of our own BF16 logits (exact);
  * our logits' rel-l2 to the reference (median and worst over the run) is at
    most LOGIT_FLOOR_X times the oracle's; cosine above LOGIT_COS;
  * our token equals the reference's, or the two tokens are a near-tie in the
    reference's own logits: a gap of at most FLIP_ULPS BF16 ulps of the top
    logit, or of at most the oracle's own largest flip gap in the run;
    at most max(MAX_FLIPS, 2 x the oracle's flips) such steps.
Free-running run: our engine's own greedy continuation equals the reference's
token for token up to the first step where the teacher-forced run flipped.
After the run the GatedDeltaNet states of every linear-attention layer are as
close to the reference's as the oracle's (within LOGIT_FLOOR_X).
"""

import math

import pytest
import torch

from parity import cosine, rel_l2

pytestmark = pytest.mark.gpu

PROMPT, NEW = 128, 300
LOGIT_COS = 0.998
LOGIT_FLOOR_X = 1.5
FLIP_ULPS = 4
MAX_FLIPS = 6


def bf16_ulp(v: float) -> float:
    """Spacing of BF16 numbers at |v| (8 significant bits)."""
    return 2.0 ** (math.floor(math.log2(max(abs(v), 1e-30))) - 7)


@pytest.fixture(scope="module")
def setup():
    from conftest import REF_LIB
    import os
    if not os.path.exists(os.path.join(REF_LIB, "libref_fused.so")):
        pytest.skip("reference kernels not built (oracle/Makefile)")
    from oracle.model import OracleModel
    from oracle.ref_engine import ReferenceKernelEngine
    from qwen35_b200.config import qwen35_4b
    from qwen35_b200.step import Qwen35StepEngine
    from qwen35_b200.weights import random_weights
    cfg = qwen35_4b()
    w = random_weights(cfg, seed=0, device="cuda")
    max_seq = PROMPT + NEW + 8
    ref = ReferenceKernelEngine(cfg, w, max_seq=max_seq)
    eng = Qwen35StepEngine(cfg, w, max_seq=max_seq, keep_logits=True)
    orc = OracleModel(cfg, w, max_seq=max_seq, device="cuda")
    prompt = torch.randint(0, cfg.vocab_size, (PROMPT,), generator=torch.Generator().manual_seed(2024)).tolist()
    # teacher-forced pass: the reference's greedy sequence drives both engines
    rows = []
    tok = prompt[0]
    ref_tokens = []
    for step in range(PROMPT + NEW):
        if step < PROMPT:
            tok = prompt[step]
        ours = eng.decode(tok)
        ol = eng.logits.clone()
        rl, rt = ref.step(tok)
        xl, xt = orc.step(tok)
        rows.append(dict(step=step, ours=ours, ref=rt, orc=xt, rel_l2=rel_l2(ol, rl), cos=cosine(ol, rl),
                         orc_rel_l2=rel_l2(xl, rl), own_argmax=int(torch.argmax(ol.float())),
                         gap=float(rl.float()[rt] - rl.float()[ours]), orc_gap=float(rl.float()[rt] - rl.float()[xt]),
                         top=float(rl.float().max())))
        if step >= PROMPT - 1:
            ref_tokens.append(rt)
        tok = rt
    torch.cuda.synchronize()
    states = {i: (eng.gdn_state(i).clone(), ref.state[i].clone(), orc.state[i].clone()) for i in ref.state}
    # free-running pass of our engine
    eng.reset()
    ours_free, _ = eng.generate(prompt, NEW)
    return dict(rows=rows, ref_tokens=ref_tokens[:NEW], ours_free=ours_free, states=states)


def test_fused_argmax_is_argmax_of_own_logits(setup):
    bad = [r for r in setup["rows"] if r["ours"] != r["own_argmax"]]
    assert not bad, bad[:3]


def _median(v):
    v = sorted(v)
    return v[len(v) // 2]


def test_logits_follow_reference(setup):
    """Our logits are as close to the reference's as the oracle's exact-dequant
    restatement is (the network amplifies every rounding difference alike)."""
    rows = setup["rows"]
    ours = [r["rel_l2"] for r in rows]
    orc = [r["orc_rel_l2"] for r in rows]
    worst_cos = min(r["cos"] for r in rows)
    print(f"\nlogits rel-l2 vs reference over {len(rows)} steps: ours median {_median(ours):.3e} max {max(ours):.3e}; "
          f"oracle median {_median(orc):.3e} max {max(orc):.3e}; our worst cosine {worst_cos:.6f}")
    assert _median(ours) <= LOGIT_FLOOR_X * _median(orc)
    assert max(ours) <= LOGIT_FLOOR_X * max(orc)
    assert worst_cos > LOGIT_COS


def test_greedy_tokens_teacher_forced(setup):
    rows = setup["rows"][PROMPT - 1:]
    flips = [r for r in rows if r["ours"] != r["ref"]]
    orc_flips = [r for r in rows if r["orc"] != r["ref"]]
    worst_orc = max([r["orc_gap"] / bf16_ulp(r["top"]) for r in orc_flips], default=0.0)
    print(f"\n{len(flips)} flips in {len(rows)} greedy steps (oracle: {len(orc_flips)} flips, "
          f"largest reference gap {worst_orc:.2f} ulp)")
    for r in flips:
        ulps = r["gap"] / bf16_ulp(r["top"])
        print(f"flip at step {r['step']}: ours {r['ours']} ref {r['ref']} reference gap {r['gap']:.4g} "
              f"({ulps:.2f} ulp of the top logit {r['top']:.4g})")
        assert ulps <= max(FLIP_ULPS, worst_orc), r
    assert len(flips) <= max(MAX_FLIPS, 2 * len(orc_flips))


def test_free_running_greedy_matches_until_first_near_tie(setup):
    rows = setup["rows"][PROMPT - 1:]
    first_flip = next((i for i, r in enumerate(rows) if r["ours"] != r["ref"]), len(rows))
    ref_tokens, ours = setup["ref_tokens"], setup["ours_free"]
    n = min(first_flip, NEW)
    agree = next((i for i in range(NEW) if ours[i] != ref_tokens[i]), NEW)
    print(f"\nfree-running: identical for the first {agree} of {NEW} tokens (first teacher-forced flip at {first_flip})")
    assert ours[:n] == ref_tokens[:n]


def test_gdn_states_follow_reference(setup):
    worst, worst_orc = 0.0, 0.0
    for i, (s_ours, s_ref, s_orc) in setup["states"].items():
        worst = max(worst, rel_l2(s_ours, s_ref))
        worst_orc = max(worst_orc, rel_l2(s_orc, s_ref))
    print(f"\nGatedDeltaNet states after {PROMPT + NEW} tokens, worst layer rel-l2 vs reference: ours {worst:.3e}, "
          f"oracle {worst_orc:.3e}")
    assert worst <= LOGIT_FLOOR_X * worst_orc
