"""NF4 frozen base (load_in_4bit; reference: micro_engram/train/model.py:122-130 through
bitsandbytes, with micro_engram/train/vendor/fsdp2_4bit.py keeping the quant state through FSDP).

Every decoder layer's four projection matrices (fused q/k/v, fused gate/up, o, down) are
stored as NF4: 4-bit codes (two per byte) and one fp32 absmax per 64 weights, 0.5625 bytes a
weight instead of 2. A layer expands its weights to bf16 just before it runs (forward, the
recompute of a checkpointed layer, and its backward) into ONE expansion buffer per device that
every layer shares, so the bf16 footprint is a single layer. Which layer the buffer holds is
tracked, so a layer never runs on another layer's weights. The 16 NF4 levels are the data
type of Dettmers et al. 2023 (QLoRA), appendix E.
"""
import torch

NF4_LEVELS = torch.tensor([-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                           -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                           0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
                           0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0])
BLOCK = 64


# ------------------------------------------------------------------ reference (CPU) codec
def quantize_ref(w):
    """(codes uint8 [numel/2], absmax fp32 [numel/64]) of a weight (numel % 64 == 0)."""
    x = w.detach().float().reshape(-1, BLOCK)
    absmax = x.abs().amax(1)
    inv = torch.where(absmax > 0, 1.0 / absmax, torch.zeros_like(absmax))
    y = x * inv[:, None]
    idx = (y[..., None] - NF4_LEVELS.to(y.device)).abs().argmin(-1).to(torch.uint8)  # first minimum wins
    idx = idx.reshape(-1, 2)
    return (idx[:, 0] | (idx[:, 1] << 4)).contiguous(), absmax.contiguous()


def dequant_ref(codes, absmax, shape, dtype=torch.bfloat16):
    lo, hi = codes & 15, codes >> 4
    idx = torch.stack([lo, hi], 1).reshape(-1).long()
    vals = NF4_LEVELS.to(codes.device)[idx].reshape(-1, BLOCK) * absmax[:, None]
    return vals.reshape(shape).to(dtype)


def quantize(w):
    if w.is_cuda and w.dtype == torch.bfloat16:
        from .. import native

        return tuple(native().nf4_quantize(w.to(torch.bfloat16).contiguous()))
    return quantize_ref(w)


def dequant_into(codes, absmax, out):
    if out.is_cuda and out.dtype == torch.bfloat16:
        from .. import native

        native().nf4_dequant(codes, absmax, out)
    else:
        out.copy_(dequant_ref(codes, absmax, out.shape, out.dtype))


# ------------------------------------------------------------------ model integration
def fused_enabled(device):
    """Whether CUDA layers run their projections on the GEMM that dequantises NF4 in-kernel
    (MICRO_ENGRAM_NF4_FUSED=1). Off by default: with training-size M (8192 tokens) every 256-row
    M tile dequantises the same weights again and the 16-level lookup costs several instructions
    per weight, far more than the tensor cores' appetite, so the layer is expanded once instead
    (into a double-buffered scratch, the next layer on a side stream; see Scratch). The in-kernel
    form pays off for small M (a few hundred tokens), where one pass over the weights dominates."""
    import os

    return device.type == "cuda" and os.environ.get("MICRO_ENGRAM_NF4_FUSED", "0") == "1"


class NF4Weights:
    """The NF4 copies of one layer's projections and the shared expansion buffer they use.
    With `fused` the tcgen05 GEMM reads the codes directly and the buffer is never filled."""

    NAMES = ("qkv", "gate_up", "o", "down")

    def __init__(self, layer, scratch):
        self.scratch = scratch
        self.packed = {}
        self.shapes = {}
        for name, w in zip(self.NAMES, _weights(layer)):
            self.shapes[name] = tuple(w.shape)
            self.packed[name] = quantize(w)
        self.fused = fused_enabled(_weights(layer)[0].device)

    def operand(self, name):
        """(codes, absmax, rows, cols) of one projection, the NF4 GEMM's B operand."""
        codes, absmax = self.packed[name]
        rows, cols = self.shapes[name]
        return codes, absmax, rows, cols

    def nbytes(self):
        return sum(c.numel() + a.numel() * 4 for c, a in self.packed.values())


class Scratch:
    """Expansion buffers per device (the weights' dtype, bf16 in training), each big enough for
    the largest layer. On CUDA there are two: a layer runs out of one while the next layer (in the
    direction of travel: +1 forward, -1 backward) is expanded into the other on a side stream, so
    the expansion overlaps the running layer's GEMMs. `owner[slot]` is the layer a slot holds
    (a layer never runs on another layer's weights) and `ready[slot]` the event of an expansion
    still pending on the side stream."""

    def __init__(self, device, numel, dtype=torch.bfloat16):
        slots = 2 if device.type == "cuda" else 1
        self.bufs = [torch.empty(numel, dtype=dtype, device=device) for _ in range(slots)]
        self.owner = [None] * slots
        self.ready = [None] * slots
        self.layers = []  # every quantized layer, in model order
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    @property
    def buf(self):
        return self.bufs[0]

    def views(self, shapes, slot=0):
        out, off = {}, 0
        for name in NF4Weights.NAMES:
            n = 1
            for s in shapes[name]:
                n *= s
            off = (off + 7) // 8 * 8  # 16-byte aligned starts for the vector kernel
            out[name] = self.bufs[slot][off:off + n].view(shapes[name])
            off += n
        return out

    def slot_of(self, layer):
        return next((i for i, o in enumerate(self.owner) if o is layer), None)


def _weights(layer):
    return (layer.qkv_weight, layer.gate_up_weight, layer.self_attn.o_proj.weight, layer.mlp.down_proj.weight)


def _need(shapes):
    return sum((-(-s[0] * s[1] // 8)) * 8 + 8 for s in shapes.values())


def _link(layer, views):
    layer.qkv_weight = views["qkv"]
    layer.gate_up_weight = views["gate_up"]
    layer.self_attn.o_proj.weight.data = views["o"]
    layer.mlp.down_proj.weight.data = views["down"]
    layer._relink()


def _expand(nf, layer, slot):
    for name, view in nf.scratch.views(nf.shapes, slot).items():
        codes, absmax = nf.packed[name]
        dequant_into(codes, absmax, view)
    nf.scratch.owner[slot] = layer


def materialize(layer, force=False, direction=1):
    """Make this layer's bf16 weights readable (its weight attributes point at the slot that holds
    them), expanding them now unless a prefetch already did; then start expanding the next layer
    in `direction` into the other slot on the side stream. No-op when the layer's GEMMs read the
    NF4 codes themselves, unless `force` (the PyTorch path)."""
    nf = getattr(layer, "_nf4", None)
    if nf is None or (nf.fused and not force):
        return
    sc = nf.scratch
    slot = sc.slot_of(layer)
    if slot is None:  # not prefetched: expand in order on the current stream
        slot = 1 if len(sc.bufs) > 1 and sc.ready[1] is None and sc.owner[0] is not None else 0
        if sc.ready[slot] is not None:  # a prefetch into this slot is still pending
            torch.cuda.current_stream().wait_event(sc.ready[slot])
        _expand(nf, layer, slot)
        sc.ready[slot] = None
    elif sc.ready[slot] is not None:
        torch.cuda.current_stream().wait_event(sc.ready[slot])
        sc.ready[slot] = None
    _link(layer, sc.views(nf.shapes, slot))
    if sc.stream is None or len(sc.bufs) < 2:
        return
    nxt_i = nf.index + direction
    if not 0 <= nxt_i < len(sc.layers):
        return
    nxt, other = sc.layers[nxt_i], 1 - slot
    if sc.owner[other] is nxt:
        return
    # every kernel of the layer that last used the other slot is queued on the current stream
    # before this point; the side stream starts after them
    sc.stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(sc.stream):
        _expand(nxt._nf4, nxt, other)
        ev = torch.cuda.Event()
        ev.record(sc.stream)
    sc.ready[other] = ev


def quantize_model_nf4(model):
    """Replace every decoder layer's projection weights with NF4 + a shared expansion buffer.
    Returns (bytes of NF4 storage, bytes freed)."""
    from .gemma import text_of

    text = text_of(model)
    layers = list(text.layers)
    if not layers:
        return 0, 0
    dev = layers[0].qkv_weight.device
    shapes = [{n: tuple(w.shape) for n, w in zip(NF4Weights.NAMES, _weights(l))} for l in layers]
    for s in shapes:
        for n, shp in s.items():
            if (shp[0] * shp[1]) % BLOCK:
                raise ValueError(f"NF4 needs weights with a multiple of 64 elements; {n} is {shp}")
    scratch = Scratch(dev, max(_need(s) for s in shapes), layers[0].qkv_weight.dtype)
    stored = freed = 0
    for i, (layer, s) in enumerate(zip(layers, shapes)):
        nf = NF4Weights(layer, scratch)
        nf.index = i
        stored += nf.nbytes()
        freed += sum(w.numel() * w.element_size() for w in _weights(layer))
        # the layer's weight attributes now alias a shared buffer; _relink keeps q/k/v and
        # gate/up views into the fused buffers
        _link(layer, scratch.views(s))
        layer._nf4 = nf
        scratch.layers.append(layer)
    if dev.type == "cuda":
        torch.cuda.empty_cache()
    return stored, freed
