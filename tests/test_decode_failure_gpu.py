"""Failure detection of the persistent decode engine without a GPU fault.

Every exchange wait of the engine is bounded: when a producer never publishes, the
waiting CTAs give up, record a status in the decode state, raise the engine's
abort flag, drain their weight copies and return, and the host call fails with
LSX_E_CUDA naming that status (the reference's analogue is a budget that expires,
Deadline / BudgetExpired, src/diagnosis.rs:22-48).  The test hook
LSX_DECODE_FAULT_TEST="cta,step,cycles" makes one CTA withhold its argmax partial
at one step and shortens the wait limit, so the other CTAs' bounded waits run out;
nothing faults, traps or spins without a limit.  The same model then generates
correctly on the same context."""
import numpy as np
import pytest

import laplacesscissors_b200 as lsx
from conftest import GOLDEN
from laplacesscissors_b200 import synth

pytestmark = pytest.mark.gpu


def test_withheld_partial_ends_in_status_and_context_recovers(gpu, oracle, monkeypatch):
    root = GOLDEN / "tiny_qwen3"
    model = lsx.Model.load(root, gpu, 32)
    assert model.fused and model.info().persistent
    prompt = synth.prompt_tokens(11, 5, 512)
    ref_tokens, _ = oracle.OracleModel(root, 32).generate(prompt, 6)

    # CTA 3 withholds its partial at step 2; waits give up after 2e7 cycles (~10 ms)
    monkeypatch.setenv("LSX_DECODE_FAULT_TEST", "3,2,20000000")
    with pytest.raises(lsx.LsxError) as err:
        model.generate(prompt, 6)
    assert err.value.status == 3  # LSX_E_CUDA
    assert "decode kernel reported status" in str(err.value)

    monkeypatch.delenv("LSX_DECODE_FAULT_TEST")
    model.reset()
    tokens, _, _ = model.generate(prompt, 6)
    assert [int(t) for t in tokens] == ref_tokens
    # and once more, from a fresh cursor, through the single-step entry
    model.reset()
    for t in prompt[:-1]:
        model.advance_token(int(t))
    assert model.advance_token(int(prompt[-1])) == ref_tokens[0]
