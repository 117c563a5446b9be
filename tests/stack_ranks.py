"""One rank of the sharded decode stack on the GPU (launched by tests/test_stack_multigpu.py
under torchrun): runs the tiny and a 2-layer 70B-shaped stack with each exchange (NCCL
all-gathers; the CUDA-core matvec's own push over peer mappings; chains of the warp-MMA kernel
pushing to peer memory, ordered by counters), one token eagerly and two more
replayed from a CUDA graph, each token on new input, and checks the logits on every rank
against the unsharded CPU reference."""
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
    refs = {}
    for exchange in ("nccl", "push", "push-split", "chain"):
        for name, cfg in (("tiny", st.CONFIGS["tiny"]), ("70b-2", dataclasses.replace(st.CONFIGS["70b"], layers=2))):
            xs = [np.random.default_rng(3 + t).standard_normal(cfg.hidden).astype(np.float32) for t in range(3)]
            for t, x in enumerate(xs):
                if (name, t) not in refs:
                    refs[name, t] = st.reference_logits(cfg, x)
            stream = torch.cuda.Stream()
            s = st.make_cuda_stack(cfg, kernels, rank, world, stream=stream, push=exchange.startswith("push"),
                                   chain=exchange == "chain", split_k=exchange == "push-split")
            s.buf["x"].copy_(torch.from_numpy(xs[0]).cuda())
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                s.forward()
            torch.cuda.synchronize()
            out = [s.buf["logits"].cpu().numpy()]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                s.forward()
            for x in xs[1:]:
                s.buf["x"].copy_(torch.from_numpy(x).cuda())
                torch.cuda.synchronize()
                g.replay()
                torch.cuda.synchronize()
                out.append(s.buf["logits"].cpu().numpy())
            g.reset()
            del g
            try:
                kernels.device_error()
            except kb.Error as e:  # keep taking the collective steps; fail at the end
                print(f"rank {rank}: {e}", flush=True)
                ok = False
            if exchange != "nccl":
                s.be.close()
            for t, y in enumerate(out):
                ref = refs[name, t]
                tol = 1e-4 * np.abs(ref).max()
                err = np.abs(y - ref).max()
                good = err <= tol
                print(f"rank {rank}/{world} {exchange} {name} token {t}: max|err| {err:.3e} (tol {tol:.3e})",
                      flush=True)
                ok = ok and good
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    kernels.close()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
