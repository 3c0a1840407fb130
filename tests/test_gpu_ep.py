"""GPU parity of the expert-parallel layer (smoe_cuda_moe_layer_ep): one
process per GPU over 2, 4 and 8 GPUs (as many as present), both layer shapes
(Qwen3-30B-A3B and Qwen3-235B-A22B), exchange inside the layer
kernel over NVLink, results against the CPU oracle of the whole layer; and
the 235B layer at batch 32 (BASELINE config 3's batched case) as expert
shards on the grouped path combined by an NCCL reduce.
Skipped on a box with a single GPU (ranks that wait on each other never run
as processes sharing one GPU)."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,fmt,shape", [(2, 1, "30b"), (2, 0, "30b"), (4, 1, "30b"), (8, 1, "30b"),
                                             (2, 1, "235b"), (4, 1, "235b"), (8, 1, "235b"),
                                             (2, 1, "235b-b32"), (4, 0, "235b-b32"), (8, 1, "235b-b32")])
def test_moe_layer_expert_parallel(world, fmt, shape):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_worker.py"), str(r), str(world),
                               str(port), str(fmt), shape], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            pytest.fail("expert-parallel ranks did not finish")
        outs.append((p.returncode, out))
    for r, (rc, out) in enumerate(outs):
        assert rc == 0, f"rank {r} failed:\n{out[-3000:]}"
