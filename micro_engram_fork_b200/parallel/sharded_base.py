"""Row-sharded frozen decoder layers (base_placement: sharded): FSDP2's memory layout for a
frozen base, with the layer all-gather carried inside the tcgen05 GEMMs.

Each rank keeps rows [r * per, (r + 1) * per) (per = ceil(rows / world)) of every layer's four
projection matrices (fused q/k/v, o, fused gate/up, down) in one symmetric buffer that every
peer maps over NVLink (CUDA IPC). A layer runs on full weights held in one of two per-GPU
gather slots (layer L in slot L % 2), which it re-reads from the peers' shards every time it
runs: the forward, and again the backward (FSDP's reshard_after_forward). So a GPU holds its
1/world share of the base plus two layers.

The all-gather of the next layer (L + 1 in the forward, L - 1 in the backward) is split into
ranges in proportion to the GEMM work of the current layer, and every tcgen05 GEMM the layer
launches copies one range in its side-copy warp (plain 16-byte peer loads into the local slot,
csrc/gather.cuh) while its tensor cores work: the collective costs no kernel of its own and
no idle SMs, and the next layer's GEMMs read their weights from local memory with TMA (a
peer's memory is never a TMA or library-GEMM operand). Whatever no GEMM carried (the first
layer of a pass, or rounding) runs as a standalone gather kernel before the layer starts.
Stream order (one stream) makes each slot's data complete before its next reader.

Reference counterpart: FSDP2 wrapping of the HF base with reshard_after_forward
(micro_engram/train/model.py:259-285, micro_engram/train/loop.py:181-194 in
Ready-Art/micro_engram_fork), whose all-gathers are separate NCCL collectives.
"""
import torch
import torch.distributed as dist

from .. import native
from .symm import SymmBuffer

MATRICES = ("qkv", "o", "gate_up", "down")


def _layer_weights(layer):
    return {"qkv": layer.qkv_weight, "o": layer.self_attn.o_proj.weight, "gate_up": layer.gate_up_weight,
            "down": layer.mlp.down_proj.weight}


def _bind(layer, views):
    layer.qkv_weight = views["qkv"]
    layer.gate_up_weight = views["gate_up"]
    layer.self_attn.o_proj.weight.data = views["o"]
    layer.mlp.down_proj.weight.data = views["down"]
    layer._relink()


def _align(n, a=256):
    return (n + a - 1) // a * a


class ShardedBase:
    def __init__(self, layers, rank, world, device, group=None):
        self.layers = list(layers)
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.shapes = [{m: tuple(w.shape) for m, w in _layer_weights(l).items()} for l in self.layers]
        self.dtype = self.layers[0].qkv_weight.dtype
        esz = torch.empty((), dtype=self.dtype).element_size()
        for shp in self.shapes:
            for m, (rows, cols) in shp.items():
                if (cols * esz) % 16:
                    raise ValueError(f"sharded base: {m} rows must be a multiple of 16 bytes ({cols} columns)")
        # shard buffer: (layer, matrix) regions of per x cols, the same offsets on every rank
        self.shard_off, off = [], 0
        for shp in self.shapes:
            offs = {}
            for m in MATRICES:
                rows, cols = shp[m]
                offs[m] = off
                off += _align(-(-rows // world) * cols * esz)
            self.shard_off.append(offs)
        self.buf = SymmBuffer(off, self.device, group)
        # slot layout of every layer's full matrices
        self.slot_off = []
        slot_bytes = 0
        for shp in self.shapes:
            offs, o = {}, 0
            for m in MATRICES:
                rows, cols = shp[m]
                offs[m] = o
                o += _align(rows * cols * esz)
            self.slot_off.append(offs)
            slot_bytes = max(slot_bytes, o)
        self.slots = [torch.empty(slot_bytes // esz, dtype=self.dtype, device=self.device) for _ in range(2)]
        self.esz = esz
        self.held = [None, None]      # layer index a slot holds (fully or in part)
        self.covered = [0, 0]         # 16-byte units of that layer's job already launched
        self.segs = {}                # (layer, slot) -> int64 [n, 4] segment table on the device
        self.total16 = [sum(rows * cols * esz // 16 for rows, cols in shp.values()) for shp in self.shapes]
        self.carry = None             # [layer, slot, next unit, end unit, per-unit weight share]
        self._take_own_rows()

    # ------------------------------------------------------------------ setup
    def _take_own_rows(self):
        """Copy this rank's rows of every layer into the shard buffer and let go of the full
        matrices (each layer then points at a gather slot until it runs)."""
        for i, layer in enumerate(self.layers):
            for m, w in _layer_weights(layer).items():
                rows, cols = self.shapes[i][m]
                per = -(-rows // self.world)
                lo, hi = min(self.rank * per, rows), min((self.rank + 1) * per, rows)
                dst = self.buf.view(self.shard_off[i][m], (per, cols), self.dtype)
                dst[:hi - lo].copy_(w.detach()[lo:hi])
            _bind(layer, self.views(i, i % 2))
            layer._sharded = self
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier()  # every rank's shards are in place before anyone gathers
        torch.cuda.empty_cache()

    def views(self, i, slot):
        out = {}
        for m in MATRICES:
            rows, cols = self.shapes[i][m]
            start = self.slot_off[i][m] // self.esz
            out[m] = self.slots[slot][start:start + rows * cols].view(rows, cols)
        return out

    def _segments(self, i, slot):
        key = (i, slot)
        table = self.segs.get(key)
        if table is not None:
            return table
        base = self.slots[slot].data_ptr()
        rows_of = []
        start16 = 0
        for m in MATRICES:
            rows, cols = self.shapes[i][m]
            per = -(-rows // self.world)
            for r in range(self.world):
                lo, hi = min(r * per, rows), min((r + 1) * per, rows)
                n16 = (hi - lo) * cols * self.esz // 16
                if n16 == 0:
                    continue
                src = self.buf.peer_addr(r, self.shard_off[i][m])
                dst = base + self.slot_off[i][m] + lo * cols * self.esz
                rows_of.append((src, dst, start16, n16))
                start16 += n16
        table = torch.tensor(rows_of, dtype=torch.int64, device=self.device)
        self.segs[key] = table
        return table

    # ------------------------------------------------------------------ per layer
    def materialize(self, layer, direction):
        """Before layer `layer` runs: make its full weights local (whatever the previous GEMMs
        did not carry is gathered now), point it at them, and hand the next layer's gather
        (`direction` +1 in the forward, -1 in the backward) to this layer's GEMMs."""
        i = layer.idx
        slot = i % 2
        if self.held[slot] != i:
            self.held[slot], self.covered[slot] = i, 0
            if self.carry is not None and self.carry[1] == slot:
                self.carry = None
        if self.covered[slot] < self.total16[i]:
            if self.carry is not None and self.carry[0] == i:
                self.carry = None
            native().layer_gather(self._segments(i, slot), self.covered[slot], self.total16[i])
            self.covered[slot] = self.total16[i]
        _bind(layer, self.views(i, slot))
        nxt = i + direction
        if 0 <= nxt < len(self.layers):
            nslot = nxt % 2
            if self.held[nslot] != nxt:
                self.held[nslot], self.covered[nslot] = nxt, 0
            if self.covered[nslot] < self.total16[nxt]:
                weights = sum(r * c for r, c in self.shapes[i].values())
                self.carry = [nxt, nslot, self.covered[nslot], self.total16[nxt],
                              (self.total16[nxt] - self.covered[nslot]) / weights]
            else:
                self.carry = None
        else:
            self.carry = None

    def take_carry(self, weight_numel):
        """The share of the pending next-layer gather that a GEMM over a weight of
        `weight_numel` elements carries: (segment table, begin16, end16) or None."""
        c = self.carry
        if c is None:
            return None
        nxt, nslot, begin, end, per_weight = c
        stop = min(end, begin + int(per_weight * weight_numel) + 1)
        self.covered[nslot] = stop
        if stop >= end:
            self.carry = None
        else:
            c[2] = stop
        return self._segments(nxt, nslot), begin, stop

    def nbytes(self):
        return self.buf.nbytes + sum(s.numel() * self.esz for s in self.slots)

    def close(self):
        self.buf.close()


def carry_into_next_gemm(weight):
    """Hand the next tcgen05 GEMM (about to run over `weight`, a layer weight of a sharded base)
    its share of the pending all-gather. No-op for other weights."""
    sb = _active()
    if sb is None:
        return
    job = sb.take_carry(weight.numel())
    if job is not None:
        segs, begin, end = job
        native().gemm_carry_copy(sb.dev, segs.data_ptr(), segs.shape[0], begin, end)


_ACTIVE = []


def _active():
    return _ACTIVE[-1] if _ACTIVE else None


def activate(sb):
    """Make `sb` the sharded base whose gathers the GEMM wrappers carry."""
    _ACTIVE.clear()
    if sb is not None:
        _ACTIVE.append(sb)
