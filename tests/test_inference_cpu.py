"""Full-recompute greedy decoding on the CPU oracle path."""
import torch

from trainium_frontier_b200.config import preset
from trainium_frontier_b200.inference.generate import generate_reference
from trainium_frontier_b200.models.gpt import GPT


def test_generate_reference_shapes_and_determinism():
    cfg = preset("tiny", depth=2)
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    p = torch.randint(1, 8192, (2, 16))
    a = generate_reference(m, p, 5)
    b = generate_reference(m, p, 5)
    assert a.shape == (2, 5) and torch.equal(a, b)
