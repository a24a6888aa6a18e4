"""YAML keys of the engram (pydantic), shared by the trainer config.

Same keys and defaults as the reference (micro_engram/args.py:1-66), so existing YAMLs load
unchanged. `micro_engram_memory_snapshot` is implemented here (the reference declares it
but never uses it): the trainer records CUDA allocations for that many steps and writes
output_dir/memory_snapshot/rank<R>_step<S>.pickle.
"""
from typing import Dict, List, Literal, Optional

from pydantic import BaseModel

Gate = Literal["scalar", "ple", "scalar_sqrt"]


class MicroEngramExtraArgs(BaseModel):
    """One more engram (micro_engram_extra); unset sizes/gate copy the main engram's."""
    layer: int
    table_size: Optional[int] = None
    table_sizes: Optional[Dict[int, Optional[int]]] = None
    dim: Optional[int] = None
    heads: Optional[int] = None
    gate: Optional[Gate] = None
    seed: Optional[int] = None          # default 10007 * layer
    init_from: Optional[str] = None     # a trained engram (output/checkpoint folder, config or weights)
    frozen: bool = False                # load but don't train (needs init_from)


class MicroEngramArgs(BaseModel):
    micro_engram_layer: int = 0
    micro_engram_table_size: int = 65_536
    micro_engram_table_sizes: Optional[Dict[int, Optional[int]]] = None
    micro_engram_dim: int = 128
    micro_engram_heads: int = 4
    micro_engram_save_steps: int = 250                # kept so old YAMLs load; unused
    micro_engram_canon_path: Optional[str] = None
    micro_engram_gate: Gate = "scalar"
    micro_engram_save_trainable_only: bool = False    # kept so old YAMLs load; unused
    micro_engram_stats_steps: int = 10
    micro_engram_seed: Optional[int] = None
    micro_engram_init_from: Optional[str] = None
    micro_engram_frozen: bool = False
    micro_engram_extra: Optional[List[MicroEngramExtraArgs]] = None
    micro_engram_lr_epoch_decay: Optional[float] = None
    micro_engram_dtype: Optional[Literal["bf16", "fp32"]] = None
    micro_engram_memory_snapshot: Optional[int] = None
    micro_engram_optimizer: Optional[Literal["lazy_adam", "rowwise_adam"]] = None
    micro_engram_sharding: Optional[Literal["rows"]] = None
    micro_engram_stochastic_rounding: bool = True
