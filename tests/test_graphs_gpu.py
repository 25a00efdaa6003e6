"""CUDA-graph training steps (minidist.GraphedStep) against the same steps run eagerly."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _train(graph: bool, batches, lr_change_at: int):
    import minidist as md
    from minidist.models import GPT, GPTConfig
    from minidist.optim import FusedAdamW

    cfg = GPTConfig(vocab_size=1000, block_size=128, n_layer=2, n_head=4, n_embd=256, seed=3)
    model = GPT(cfg, device=torch.device("cuda"))
    opt = FusedAdamW(model.parameters(), lr=1e-3, capturable=graph)

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
            loss = model(x, y)[1]
        loss.backward()
        opt.step()
        return loss

    losses = []
    if graph:
        run = md.GraphedStep(step, batches[0], warmup=2, optimizers=[opt])
    else:
        step(*batches[0])
        step(*batches[0])
        run = step
    for i, b in enumerate(batches[1:]):
        if i == lr_change_at:
            opt.param_groups[0]["lr"] = 3e-4
        losses.append(float(run(*b).item()))
    w = model.blocks[0].attn.qkv.weight.detach().clone()
    sd_step = None
    if graph:
        sd_step = float(opt.state_dict()["state"][0]["step"])
        run.release()
    return losses, w, sd_step


def test_graphed_step_matches_eager():
    g = torch.Generator().manual_seed(5)
    batches = [(torch.randint(0, 1000, (4, 128), generator=g).cuda(),
                torch.randint(0, 1000, (4, 128), generator=g).cuda()) for _ in range(7)]
    eager, w_e, _ = _train(False, batches, lr_change_at=3)
    graphed, w_g, sd_step = _train(True, batches, lr_change_at=3)
    # Same trajectory: the replayed optimizer advances its step and follows the lr change.
    for a, b in zip(eager, graphed, strict=True):
        assert abs(a - b) <= 2e-3 * abs(a), (eager, graphed)
    # AdamW turns atomic-order noise in tiny gradients into lr-sized steps, so bound the
    # element-wise difference by the steps' total learning rate, and the typical one tightly.
    total_lr = 2 * 1e-3 + 3 * 1e-3 + 3 * 3e-4
    assert (w_e - w_g).abs().max().item() <= 2 * total_lr
    assert ((w_e - w_g).abs().mean() / w_e.abs().mean()).item() < 2e-2
    assert sd_step == 2 + 6, sd_step  # 2 eager warm-up steps + 6 replays, synced from the device
    assert graphed[-1] < graphed[0]


def test_graphed_step_rejects_non_capturable_optimizer():
    import minidist as md
    from minidist.optim import FusedAdamW

    p = torch.nn.Parameter(torch.randn(16, device="cuda"))
    opt = FusedAdamW([p], lr=1e-3)
    with pytest.raises(ValueError):
        md.GraphedStep(lambda x: x, [torch.zeros(1, device="cuda")], optimizers=[opt])
