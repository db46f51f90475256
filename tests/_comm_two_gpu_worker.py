"""Worker of `test_comm_gpu.py` (torch.distributed.run, one process per GPU): the library's own NCCL C ABI
(`libhb_comm.so`) does the band halo exchange and the head-pair all-gather; results are checked exactly."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))  # only hands out the communicator id
    from hummingbird_b200 import parallel as par
    from hummingbird_b200.comm import HbComm
    comm = HbComm(rank, world, timeout_ms=30_000)
    ok = True
    # halo exchange: every row carries its global row index, two batch elements
    length, window, width = 1000, 128, 40
    lay = par.band_layout(length, world, rank, window)
    rows = torch.arange(length, dtype=torch.float32, device="cuda")[None, :, None].repeat(2, 1, width)
    rows[1] += 10_000
    buf = torch.full((2, lay["rows"], width), -1.0, device="cuda")
    buf[:, lay["before"]:lay["before"] + lay["q_count"]] = rows[:, lay["s0"]:lay["s1"]]
    comm.halo_exchange(buf, lay)
    torch.cuda.synchronize()
    ok &= torch.equal(buf, rows[:, lay["pos0"]:lay["pos0"] + lay["rows"]])
    # head-pair gather, uneven split of 5 pairs
    pairs = 5
    p0, p1 = par.shard_pairs(pairs, world, rank)
    local = torch.arange(p0 * 128, p1 * 128, dtype=torch.float32, device="cuda").to(torch.bfloat16).repeat(2, 3, 1)
    full = comm.gather_pairs(local, pairs)
    torch.cuda.synchronize()
    ok &= torch.equal(full, torch.arange(pairs * 128, dtype=torch.float32, device="cuda").to(torch.bfloat16).repeat(2, 3, 1))
    # the host-streamed API on a sequence shard (boundary rows first, halo exchange, then the rest) against
    # the whole sequence computed on this GPU
    from hummingbird_b200 import band_attention as hb
    from hummingbird_b200.workloads import band_inputs
    w = band_inputs("cuda", seed=9, length=2000, d_model=256, heads=4, window=128)
    freqs, lam = torch.from_numpy(w.inv_freq).cuda(), torch.from_numpy(w.lam).cuda()
    full = hb.band_attention(w.qkv, w.q_norm, w.k_norm, freqs, w.heads, 64, w.window, lam=lam)
    lay = par.band_layout(2000, world, rank, 128)
    host = w.qkv[:, lay["s0"]:lay["s1"]].cpu().pin_memory()
    got = hb.band_attention_from_host(host, w.q_norm, w.k_norm, freqs, w.heads, 64, w.window, lam=lam,
                                      layout=lay, comm=comm, chunk_rows=300)
    torch.cuda.synchronize()
    ok &= torch.equal(got, full[:, lay["s0"]:lay["s1"]].cpu())
    comm.close()
    flag = torch.tensor([0 if ok else 1])
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
