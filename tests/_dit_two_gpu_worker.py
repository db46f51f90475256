"""Worker of `test_dit_two_gpu.py` (launched by torch.distributed.run, one process per GPU): one small clip's
denoise step split over the ranks (token rows + head pairs, NCCL all-to-alls, the CUDA kernels) against the
same step on one GPU."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import ClipShape, DiT
    shape = ClipShape(batch=2, latents=248, depth=2, steps=2)
    cfg = DiTConfig(ff_quant="w8a8")
    g = torch.Generator(device="cuda").manual_seed(5)
    cross = torch.randn(2, 128, 768, generator=g, device="cuda")
    glob = torch.randn(2, 768, generator=g, device="cuda")
    x = torch.randn(2, 64, 248, generator=g, device="cuda").to(torch.bfloat16)
    eps = torch.randn(2, 64, 248, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.full((2,), 0.9, device="cuda", dtype=torch.bfloat16)
    tn = torch.full((2,), 0.5, device="cuda", dtype=torch.bfloat16)
    single = DiT(cfg, shape, "cuda")
    expect = single.step(x, t, tn, eps, single.prepare_static(cross, glob)).float()
    split = os.environ.get("HB_DIT_SPLIT_BATCH", "1") == "1"
    model = DiT(cfg, shape, "cuda", group=dist.group.WORLD, split_batch=split)
    got = model.gather_latents(model.step(model.local_view(x), t, tn, model.local_view(eps),
                                          model.prepare_static(cross, glob))).float()
    rel = ((got - expect).norm() / expect.norm()).item()
    ok = got.shape == expect.shape and bool(torch.isfinite(got).all()) and rel < 2e-2
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    if rank == 0:
        print(f"world {world} relative difference {rel:.3e}")
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
