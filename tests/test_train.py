"""DDPTrainer's host-fed loop on CPU (single-process gloo): every batch is
stepped and every step's loss comes back to the host."""
import os
import socket

import torch


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_train_steps_reads_every_loss():
    import torch.distributed as dist

    from mini_nangila_b200.models import GPT2, GPT2Config
    from mini_nangila_b200.train import DDPTrainer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        torch.manual_seed(0)
        cfg = GPT2Config.tiny()
        tr = DDPTrainer(GPT2(cfg), hook="nccl", device=torch.device("cpu"), bucket_cap_mb=0.05)
        g = torch.Generator().manual_seed(1)
        batches = []
        for _ in range(4):
            t = torch.randint(0, cfg.vocab_size, (2, 17), generator=g)
            batches.append((t[:, :-1].contiguous(), t[:, 1:].contiguous()))
        losses = tr.train_steps(batches)
        assert len(losses) == 4 and all(isinstance(x, float) for x in losses)
        assert tr.steps_done == 4
    finally:
        dist.destroy_process_group()
