"""The fine-tune throughput harness (finetune_hf.py, the method of the
reference's finetune_hf.py:90-127) on a small synthetic Qwen3: both runs train
from the same weights on the same blocks, their losses stay finite and track
each other (the only difference is attention's summation order), and the
harness reports a step time for each."""
import pytest

pytestmark = pytest.mark.gpu


def test_finetune_runs_track(cuda):
    import finetune_hf
    s = finetune_hf.main(["--layers", "2", "--vocab", "4096", "--seq-len", "1024", "--steps", "5",
                          "--warmup", "1", "--blocks", "3", "--loss-chunks", "2", "--lr", "1e-4"])
    sdpa, ours = s["results"]
    assert len(sdpa["losses"]) == len(ours["losses"]) == 5
    assert all(x == x and abs(x) < 1e4 for x in sdpa["losses"] + ours["losses"])
    assert s["max_loss_difference"] < 2e-2
    assert sdpa["median_step_ms"] > 0 and ours["median_step_ms"] > 0


def test_finetune_bf16(cuda):
    import finetune_hf
    s = finetune_hf.main(["--layers", "1", "--vocab", "2048", "--seq-len", "512", "--steps", "3",
                          "--warmup", "1", "--blocks", "2", "--loss-chunks", "2", "--dtype", "bf16"])
    assert s["max_loss_difference"] < 5e-2
