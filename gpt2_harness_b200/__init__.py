"""gpt2_harness_b200: a B200-native GPT-2 distributed-training framework.

PyTorch is the framework layer (model definition, parallel strategies,
counters, checkpoints, tooling); the hot paths run on hand-written sm_100a
kernels in ``gpt2_harness_b200._C`` (built in-tree by ``setup.py``).
"""

from gpt2_harness_b200.config import GPT2_SIZES, GPTConfig, TrainConfig, gpt2_config

__all__ = ["GPTConfig", "TrainConfig", "GPT2_SIZES", "gpt2_config"]
__version__ = "0.1.0"
