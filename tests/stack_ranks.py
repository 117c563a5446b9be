"""One rank of the sharded decode stack on the GPU (launched by tests/test_stack_multigpu.py
under torchrun): runs the tiny and a 2-layer 70B-shaped stack over NCCL, eagerly and from a
CUDA graph, and checks the logits on every rank against the unsharded CPU reference."""
import dataclasses
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import kernite_b200 as kb  # noqa: E402
from kernite_b200 import stack as st  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    kernels = kb.Kernels.load(local)
    ok = True
    for name, cfg in (("tiny", st.CONFIGS["tiny"]), ("70b-2", dataclasses.replace(st.CONFIGS["70b"], layers=2))):
        x = np.random.default_rng(3).standard_normal(cfg.hidden).astype(np.float32)
        stream = torch.cuda.Stream()
        s = st.make_cuda_stack(cfg, kernels, rank, world, stream=stream)
        s.buf["x"].copy_(torch.from_numpy(x).cuda())
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            s.forward()
        torch.cuda.synchronize()
        eager = s.buf["logits"].cpu().numpy()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            s.forward()
        s.buf["logits"].zero_()
        g.replay()
        torch.cuda.synchronize()
        replay = s.buf["logits"].cpu().numpy()
        del g
        kernels.device_error()
        ref = st.reference_logits(cfg, x)
        tol = 1e-4 * np.abs(ref).max()
        good = np.abs(eager - ref).max() <= tol and np.array_equal(eager, replay)
        print(f"rank {rank}/{world} {name}: max|err| {np.abs(eager - ref).max():.3e} (tol {tol:.3e}) "
              f"graph==eager {np.array_equal(eager, replay)}", flush=True)
        ok = ok and good
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    kernels.close()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
