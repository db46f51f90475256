"""Worker of `test_comm_gpu.py`: rank 0 of a two-rank communicator whose rank 1 never joins. The library's
host-side deadline must end the initialisation with HB_ERR_TIMEOUT (no GPU work is involved)."""
import ctypes
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import torch
    torch.cuda.set_device(0)
    from hummingbird_b200 import comm
    lib = comm.lib()
    h = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(comm.unique_id(), comm.ID_BYTES)
    t0 = time.time()
    code = lib.hb_comm_init(uid, 2, 0, 2000, ctypes.byref(h))
    took = time.time() - t0
    print(f"status {code} after {took:.1f} s, handle {h.value}")
    sys.exit(0 if code == 6 and h.value is None and took < 30 else 1)


if __name__ == "__main__":
    main()
