"""vLLM plugin for micro-engram, loaded through the `vllm.general_plugins` entry point
(`micro_engram = micro_engram_vllm:register`; reference: micro_engram_vllm/__init__.py:1-17).

Registers the engram Gemma 4 classes under the stock architecture names (models without an
engram config run as plain Gemma 4), and makes the V2 runner's model state fill the engram
history buffer whichever way the installed vLLM builds that state.
"""


def register():
    import os

    from vllm import ModelRegistry

    if os.environ.get("MICRO_ENGRAM_CONFIG"):  # an engram is requested: its history needs the V2 runner
        os.environ.setdefault("VLLM_USE_V2_MODEL_RUNNER", "1")

    ModelRegistry.register_model("Gemma4ForCausalLM", "micro_engram_vllm.model:EngramGemma4ForCausalLM")
    ModelRegistry.register_model("Gemma4ForConditionalGeneration",
                                 "micro_engram_vllm.model:EngramGemma4ForConditionalGeneration")
    _wrap_model_state()


def _wrap_model_state():
    """Runners that build the model state from the architecture (init_model_state) get the
    engram fill attached to whatever state they build."""
    try:
        from vllm.v1.worker.gpu import model_runner as mr
    except Exception:  # noqa: BLE001 - no V2 runner in this vLLM: the model's get_model_state_cls is used
        return
    orig = getattr(mr, "init_model_state", None)
    if orig is None or getattr(orig, "_micro_engram", False):
        return

    def init_model_state(vllm_config, model, encoder_cache, device):
        from .model_state import attach

        return attach(orig(vllm_config, model, encoder_cache, device), model)

    init_model_state._micro_engram = True
    mr.init_model_state = init_model_state
