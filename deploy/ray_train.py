"""GPT-2 training on a Ray cluster of B200 nodes.

Every training worker is a Ray actor that owns one GPU and runs the same
entry point as torchrun (``gpt2_harness_b200.launch``) with the RANK /
WORLD_SIZE / MASTER_* environment set, so the job is identical to the Slurm
and Kubernetes recipes. Placement is ``STRICT_PACK`` per node (a node's 8
workers share its NVSwitch), and the driver restarts the whole group up to
``max_failures`` times; every restart resumes from the newest checkpoint.

    python deploy/ray_train.py --nodes 2 --gpus-per-node 8 --ckpt-dir /shared/ckpt
"""

from __future__ import annotations

import argparse
import os
import socket


def main() -> int:
    import ray
    from ray.util.placement_group import placement_group
    from ray.util.scheduling_strategies import PlacementGroupSchedulingStrategy

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--nodes", type=int, default=1)
    ap.add_argument("--gpus-per-node", type=int, default=8)
    ap.add_argument("--ckpt-dir", required=True)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--model", default="gpt2")
    ap.add_argument("--max-failures", type=int, default=3)
    ap.add_argument("--port", type=int, default=29512)
    a = ap.parse_args()
    ray.init(address=os.environ.get("RAY_ADDRESS", "auto"))
    world = a.nodes * a.gpus_per_node

    @ray.remote(num_gpus=1, num_cpus=8)
    class Worker:
        def addr(self) -> str:
            return socket.gethostbyname(socket.gethostname())

        def run(self, rank: int, master: str, argv: list) -> int:
            os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK="0", MASTER_ADDR=master,
                              MASTER_PORT=str(a.port), TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
            from gpt2_harness_b200.launch import main as launch_main
            return launch_main(argv)

    argv = ["--model", a.model, "--steps", str(a.steps), "--ckpt-dir", a.ckpt_dir,
            "--comm", "p2p" if a.nodes == 1 else "nccl"]
    for attempt in range(a.max_failures + 1):
        pgs = [placement_group([{"GPU": 1, "CPU": 8}] * a.gpus_per_node, strategy="STRICT_PACK")
               for _ in range(a.nodes)]
        ray.get([pg.ready() for pg in pgs])
        workers = [Worker.options(scheduling_strategy=PlacementGroupSchedulingStrategy(
            placement_group=pgs[r // a.gpus_per_node])).remote() for r in range(world)]
        master = ray.get(workers[0].addr.remote())
        try:
            ray.get([w.run.remote(r, master, argv) for r, w in enumerate(workers)])
            return 0
        except ray.exceptions.RayError as exc:
            print(f"attempt {attempt}: {exc!r}; restarting from the newest checkpoint")
        finally:
            for w in workers:
                ray.kill(w)
    return 1


if __name__ == "__main__":
    raise SystemExit(main())
