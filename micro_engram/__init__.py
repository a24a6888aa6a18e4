"""micro-engram on B200: a hashed n-gram memory for frozen decoder models.

Train with `torchrun -m micro_engram.train cfg.yaml` (micro_engram/train). The engram
module, weight loaders and run config are in module.py, weights.py and runconfig.py; vLLM
serving is the separate micro_engram_vllm package. The sm_100a engine underneath is
micro_engram_fork_b200.
"""
from .runconfig import CONFIG_NAME  # noqa: F401
