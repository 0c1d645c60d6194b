"""Full resume: stopping after k steps, saving, and continuing in a fresh Trainer gives the
same losses as an uninterrupted run (CPU, exact)."""
import torch


def _cfg():
    from trainium_frontier_b200.config import preset
    return preset("tiny", depth=2, progress_mode="steps", num_steps=8, device_batch_size=2,
                  total_batch_size=2 * 256 * 2, grad_sync="none")


def test_resume_is_exact(tmp_path):
    from trainium_frontier_b200.train import Trainer
    dev = torch.device("cpu")
    a = Trainer(_cfg(), dev)
    ref = [a.train_step() for _ in range(4)]
    b = Trainer(_cfg(), dev)
    first = [b.train_step() for _ in range(2)]
    assert first == ref[:2]
    b.save_resume(tmp_path / "resume_rank0.pt")
    torch.manual_seed(1234)  # disturb the global RNG: resume must restore it
    c = Trainer(_cfg(), dev)
    c.load_resume(tmp_path / "resume_rank0.pt")
    assert c.step_idx == 2
    rest = [c.train_step() for _ in range(2)]
    assert rest == ref[2:], (rest, ref[2:])
