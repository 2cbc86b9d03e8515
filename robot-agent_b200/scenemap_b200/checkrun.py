"""Checked run of the benchmark workload (config-1 box rooms, device-resident inputs).

    python robot-agent_b200/scenemap_b200/checkrun.py MAPS FRAMES MAX_OBJECTS

Pushes MAPS maps for FRAMES keyframes and, after every 16 frames, prints the device error word
and the first failed bounds check; it stops at the first nonzero one.  Bounds checks exist only
in a library built with -DSMG_CHECKS (select it with the SMG_LIB environment variable); with the
production library the check record is always zero and the run is a plain workload driver, as
used for small profiling captures.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from scenemap_b200 import smg  # noqa: E402
from scenemap_b200.workload import RoomBatch  # noqa: E402


def main(M: int, NF: int, O: int) -> None:
    wl = RoomBatch(M, 1000, NF, D=1152, bf16=True, max_det=24)
    B = smg.Batch(M, max_objects=O, emb_dim=1152, max_w=640, max_h=480, max_det=24, grid=(512, 512, -196, -206))
    for f0 in range(0, NF, 16):
        nf = min(16, NF - f0)
        R = wl.render(f0, nf, 0)
        for fi in range(nf):
            keep = []
            B.push(None, smg.SMG_MEM_DEVICE, structs=wl.structs(R, fi, keep), stream=0)
        torch.cuda.synchronize()
        print("frames", f0, f0 + nf, "err", B.error_word(), "chk", B.debug_check(), flush=True)
        assert B.error_word() == 0 and not any(B.debug_check())
    print("work", B.work())
    B.close()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))
