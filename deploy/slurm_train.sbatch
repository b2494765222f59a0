#!/bin/bash
# Multi-node GPT-2 training on B200 HGX nodes (8 GPUs each) under Slurm.
#
#   sbatch deploy/slurm_train.sbatch            # 8 nodes x 8 B200 by default
#   NODES=2 sbatch --nodes=2 deploy/slurm_train.sbatch
#
# One torchrun per node (srun), one process per GPU. The job requeues itself
# on pre-emption: Slurm sends SIGUSR1 180 s before the time limit, the
# training loop checkpoints at the next step boundary and exits, and the
# requeued job resumes from the newest checkpoint under $CKPT_DIR.
#SBATCH --job-name=gpt2-b200
#SBATCH --nodes=8
#SBATCH --ntasks-per-node=1
#SBATCH --gpus-per-node=8
#SBATCH --cpus-per-task=96
#SBATCH --exclusive
#SBATCH --time=24:00:00
#SBATCH --requeue
#SBATCH --signal=B:USR1@180
#SBATCH --output=logs/%x-%j.out

set -euo pipefail
mkdir -p logs
CKPT_DIR=${CKPT_DIR:-$PWD/ckpt/$SLURM_JOB_NAME}
DATA=${DATA:-}
MODEL=${MODEL:-gpt2}
STEPS=${STEPS:-20000}

# rendezvous: the first node of the allocation
export MASTER_ADDR=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n1)
export MASTER_PORT=${MASTER_PORT:-29511}

# NCCL over NVLink 5 / NVSwitch inside a node (NVLS in-switch reduction when
# available) and InfiniBand between nodes with GPUDirect RDMA.
export NCCL_NVLS_ENABLE=${NCCL_NVLS_ENABLE:-1}
export NCCL_IB_HCA=${NCCL_IB_HCA:-mlx5}
export NCCL_SOCKET_IFNAME=${NCCL_SOCKET_IFNAME:-^lo,docker}
export NCCL_NET_GDR_LEVEL=${NCCL_NET_GDR_LEVEL:-PHB}
export TORCH_NCCL_ASYNC_ERROR_HANDLING=1
export OMP_NUM_THREADS=8

# forward the pre-emption warning to the training processes
trap 'echo "USR1: checkpoint + requeue"; kill -USR1 $(jobs -p) 2>/dev/null || true' USR1

# The fused peer-memory all-reduce reaches peers inside one node only; across
# nodes the NCCL path carries the gradients.
COMM=p2p
if [ "${SLURM_NNODES:-1}" -gt 1 ]; then COMM=nccl; fi

srun --kill-on-bad-exit=1 bash -c "
  python -m torch.distributed.run --nnodes=\$SLURM_NNODES --nproc-per-node=8 \
    --node-rank=\$SLURM_NODEID --master-addr=$MASTER_ADDR --master-port=$MASTER_PORT \
    -m gpt2_harness_b200.launch --model $MODEL ${DATA:+--data $DATA} --steps $STEPS \
    --comm $COMM --ckpt-dir $CKPT_DIR --ckpt-every 500 --log logs/$SLURM_JOB_ID.metrics.jsonl
" &
wait
