"""One rank of the tensor-parallel decoder check (launched by test_gpu_tp.py via
torch.distributed.run): teacher-forced greedy predictions of the small decoder."""

import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, ".."), os.path.join(HERE, "..", "spark-mlx-llm_b200")]

from spark_b200.decoder import DecoderConfig, SyntheticDecoder  # noqa: E402


def predictions(world, rank, group, device, steps=24, prompt_len=8, batch=2):
    cfg = DecoderConfig.small(num_layers=3)
    dec = SyntheticDecoder(cfg, batch=batch, capacity=prompt_len + steps + 16, device=device, seed=3, rank=rank,
                           world=world, group=group)
    gen = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, cfg.vocab, (batch, prompt_len), generator=gen, dtype=torch.int32)
    forced = torch.randint(0, cfg.vocab, (steps, batch), generator=gen, dtype=torch.int32)
    dec.prefill_stepwise(prompt.to(device))  # the same prompt path at every degree
    out = []
    for s in range(steps):
        dec.tokens.copy_(forced[s].to(device))
        dec.step()
        out.append(dec.tokens.cpu().numpy().copy())
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
        dec.close()
    return np.stack(out)


def main():
    out_path = sys.argv[1]
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    try:
        pred = predictions(world, rank, dist.group.WORLD, device)
        if rank == 0:
            np.save(out_path, pred)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
