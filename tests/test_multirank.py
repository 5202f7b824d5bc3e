"""The N>1 host logic of bench.py on CPU: two `gloo` ranks as child processes (no GPU).

Under torchrun each rank forecasts its own seeded block of series (weak scaling, no collective on
the data path) and the timed figures are reduced as the maximum over ranks. These tests check
both with world size 2: the ranks' blocks are disjoint and together equal one process's block of
2·b series, and every rank reads back the slowest rank's time.
"""
import os
import socket
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import os, sys
import numpy as np
sys.path[:0] = [os.path.join(%(root)r, "tsfm-zig_b200"), %(root)r]
import torch.distributed as dist
from datetime import timedelta
import bench
from tsfm_b200 import synthetic as syn
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
dist.init_process_group("gloo", timeout=timedelta(seconds=60))
m = bench.max_over_ranks(10.0 + rank, world, "cpu")
x = syn.seeded_series(%(b)d, %(t)d, seed=bench.series_seed(rank, %(b)d))
np.save(os.path.join(%(out)r, "rank%%d.npy" %% rank), x)
with open(os.path.join(%(out)r, "rank%%d.max" %% rank), "w") as f:
    f.write(repr(m))
dist.barrier()
dist.destroy_process_group()
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_shard_series_and_take_the_slowest_time(tmp_path):
    b, t, world = 4, 96, 2
    code = CHILD % {"root": ROOT, "b": b, "t": t, "out": str(tmp_path)}
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    for p in procs:
        out, _ = p.communicate(timeout=240)
        assert p.returncode == 0, out[-2000:]

    for r in range(world):
        assert float((tmp_path / ("rank%d.max" % r)).read_text()) == 10.0 + world - 1

    sys.path[:0] = [os.path.join(ROOT, "tsfm-zig_b200"), ROOT]
    import bench
    from tsfm_b200 import synthetic as syn
    blocks = [np.load(tmp_path / ("rank%d.npy" % r)) for r in range(world)]
    whole = syn.seeded_series(b * world, t, seed=bench.series_seed(0, b))
    np.testing.assert_array_equal(np.concatenate(blocks), whole)
    assert not np.array_equal(blocks[0], blocks[1], equal_nan=True)


def test_single_rank_max_is_the_value_itself():
    sys.path[:0] = [ROOT]
    import bench
    assert bench.max_over_ranks(3.25, 1, "cpu") == 3.25
