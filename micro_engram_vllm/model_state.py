"""Model Runner V2 state that fills the engram history buffer before every step
(reference: micro_engram_vllm/model_state.py:7-32).

vLLM releases differ in how the runner picks its model state: some ask the model
(`get_model_state_cls`), others build one from the architecture (`init_model_state`). The
mixin below works for both: `EngramModelState` is the class for the first, and
`attach(state, model)` turns an already built state into an engram state for the second
(micro_engram_vllm.register installs that wrapper).
"""
from .ids import fill_engram_ids


class _EngramStateMixin:
    def _engram_setup(self, model):
        self.engram_ids = getattr(model, "micro_engram_ids", None)  # owned by the model: fixed address
        if self.engram_ids is not None and self.engram_ids.shape[0] < self.max_num_tokens:
            raise ValueError(f"[micro_engram] history buffer holds {self.engram_ids.shape[0]} tokens, the runner "
                             f"schedules up to {self.max_num_tokens}")

    def prepare_inputs(self, input_batch, req_states):
        model_inputs = super().prepare_inputs(input_batch, req_states)
        if self.engram_ids is not None:
            fill_engram_ids(self.engram_ids, input_batch.input_ids, input_batch.positions, input_batch.idx_mapping,
                            input_batch.query_start_loc, req_states.all_token_ids.gpu,
                            num_reqs=input_batch.num_reqs, num_tokens=input_batch.num_tokens,
                            num_tokens_padded=input_batch.num_tokens_after_padding)
        return model_inputs


def _default_state_cls():
    from vllm.v1.worker.gpu.model_states.default import DefaultModelState

    return DefaultModelState


class _Lazy(type):
    """Builds EngramModelState on first use, so importing this module needs no vLLM."""

    _cls = None

    def _get(cls):
        if _Lazy._cls is None:
            base = _default_state_cls()

            class EngramModelState(_EngramStateMixin, base):
                def __init__(self, vllm_config, model, encoder_cache, device):
                    super().__init__(vllm_config, model, encoder_cache, device)
                    self._engram_setup(model)

            _Lazy._cls = EngramModelState
        return _Lazy._cls

    def __call__(cls, *args, **kwargs):
        return cls._get()(*args, **kwargs)


class EngramModelState(metaclass=_Lazy):
    """DefaultModelState + the engram history fill (constructed through the metaclass)."""


def attach(state, model):
    """Make a built model state fill the engram history of `model` (no-op without an engram).

    The state's prepare_inputs is wrapped on the instance (its class may not allow a
    __class__ swap), so the runner's own state class and its other methods stay as built."""
    if getattr(model, "micro_engram_ids", None) is None or getattr(state, "_micro_engram_attached", False):
        return state
    inner = state.prepare_inputs

    def prepare_inputs(input_batch, req_states):
        model_inputs = inner(input_batch, req_states)
        fill_engram_ids(state.engram_ids, input_batch.input_ids, input_batch.positions, input_batch.idx_mapping,
                        input_batch.query_start_loc, req_states.all_token_ids.gpu, num_reqs=input_batch.num_reqs,
                        num_tokens=input_batch.num_tokens, num_tokens_padded=input_batch.num_tokens_after_padding)
        return model_inputs

    _EngramStateMixin._engram_setup(state, model)
    state.prepare_inputs = prepare_inputs
    state._micro_engram_attached = True
    return state
