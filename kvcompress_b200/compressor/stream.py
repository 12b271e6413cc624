"""Token-range decode streams over a set of JoLT payloads.

A consumer that reads the cache in blocks of tokens (an attention kernel
walking a long context, or an offload path restoring it piece by piece)
decodes every layer's K and V for tokens ``[t0, t1)``, then the next block.
The reference decodes whole payloads (``reconstruct_payload``,
kvcompress/compressor/jolt.py:401-463); here the part of the decode that does
not depend on the range (the codes' tensor maps and each cell's rotation
image) is built once per group of same-layout payloads, and each block is
one or two kernel launches per group (``ops.DecodePlan``).  Layouts without a
tensor-core plan fall back to ``decompress_tokens``'s path for every block.
"""

from __future__ import annotations

from typing import Iterator, Sequence

import torch

from kvcompress_b200 import ops
from kvcompress_b200._native import KVC
from kvcompress_b200.compressor.base import CompressedPayload
from kvcompress_b200.compressor.cells import decode_args, decompress_cells
from kvcompress_b200.compressor.jolt import group_payloads

__all__ = ["CapturedStream", "DecodeStream"]


class DecodeStream:
    """Decode tokens ``[t0, t1)`` of many JoLT payloads at once.

    ``payloads``: a list of ``(key_payload, value_payload)`` pairs (one per
    layer, as ``compress`` returns them) or a flat list of payloads.  The
    payload tensors must stay alive and unchanged while the stream is used;
    decode from one CUDA stream at a time.

    ``decode(t0, t1)`` returns the decoded tensors in the input's structure:
    ``(m, t1 - t0, d)`` per payload, bit for bit the rows
    ``JoLTCompressor.decompress_tokens`` gives for the range.
    """

    def __init__(self, payloads: Sequence):
        self._pairs = bool(payloads) and isinstance(payloads[0], (tuple, list))
        flat: list[CompressedPayload] = [p for pair in payloads for p in pair] if self._pairs else list(payloads)
        if not flat:
            raise ValueError("DecodeStream: no payloads")
        for p in flat:
            if p.method != "jolt":
                raise ValueError(f"DecodeStream decodes JoLT payloads (got method={p.method!r})")
        self._flat = flat
        self.tokens = int(flat[0].shape[1])
        if any(int(p.shape[1]) != self.tokens for p in flat):
            raise ValueError("DecodeStream: every payload must hold the same number of tokens")
        self._groups = []  # (member indices, plan or None)
        for members in group_payloads(flat):
            for i in range(0, len(members), KVC.MAX_CELLS):
                part = members[i:i + KVC.MAX_CELLS]
                shape, odt, _dev, kw = decode_args([flat[j] for j in part])
                plan = None
                if kw.get("bits", 0) > 0:
                    plan = ops.DecodePlan.make(shape, odt, codes=kw["codes"], scales=kw["scales"],
                                               zps=kw["zps"], bits=kw["bits"], symmetric=kw["symmetric"],
                                               scale_mode=kw["scale_mode"], group_size=kw["group_size"],
                                               factors=kw["factors"], proj=kw["proj"])
                self._groups.append((part, plan))

    @property
    def planned(self) -> bool:
        """True when every group decodes through a prepared plan."""
        return all(plan is not None for _, plan in self._groups)

    def decode(self, t0: int, t1: int):
        """Tokens ``[t0, t1)`` of every payload (one or two launches per group)."""
        t0, t1 = int(t0), int(t1)
        if not 0 <= t0 < t1 <= self.tokens:
            raise ValueError(f"DecodeStream.decode: bad token range [{t0}, {t1}) of {self.tokens}")
        outs: list[torch.Tensor | None] = [None] * len(self._flat)
        for members, plan in self._groups:
            rec = plan.run(t0, t1) if plan is not None else decompress_cells(
                [self._flat[j] for j in members], t0=t0, t1=t1)
            for j, r in zip(members, rec):
                outs[j] = r
        if self._pairs:
            return [(outs[2 * i], outs[2 * i + 1]) for i in range(len(outs) // 2)]
        return outs

    def capture(self, block: int) -> "CapturedStream":
        """Every block of the stream recorded as one CUDA graph.

        ``replay()`` then decodes all blocks (two kernels per block and
        group, no host work in between) into fixed output tensors,
        ``outputs[i]`` holding block i in ``decode``'s structure.  The outputs
        are overwritten by each replay.  Needs a tensor-core plan for every
        group."""
        if not self.planned:
            raise RuntimeError("DecodeStream.capture: every group needs a tensor-core plan")
        spans = [(t0, min(t0 + block, self.tokens)) for t0 in range(0, self.tokens, block)]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for t0, t1 in spans[:1]:  # warm-up outside the graph (kernel attributes, allocator)
                self.decode(t0, t1)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outputs = [self.decode(t0, t1) for t0, t1 in spans]
        return CapturedStream(graph, spans, outputs)

    def blocks(self, block: int) -> Iterator[tuple[int, int, list]]:
        """``(t0, t1, decode(t0, t1))`` for consecutive blocks of ``block`` tokens."""
        if block <= 0:
            raise ValueError("DecodeStream.blocks: block must be positive")
        for t0 in range(0, self.tokens, block):
            t1 = min(t0 + block, self.tokens)
            yield t0, t1, self.decode(t0, t1)


class CapturedStream:
    """A decode stream recorded as one CUDA graph (``DecodeStream.capture``)."""

    def __init__(self, graph: torch.cuda.CUDAGraph, spans: list[tuple[int, int]], outputs: list):
        self.graph, self.spans, self.outputs = graph, spans, outputs

    def replay(self) -> list:
        """Decode every block again into ``outputs`` (asynchronous, current stream)."""
        self.graph.replay()
        return self.outputs
