"""Packed quantized weights: the checkpoint form of a quantization result.

The reference returns only the dequantized floats (``quant.py:37``); a
deployment needs the codes, the group parameters and the act-order
permutation.  ``PackedLinear`` holds exactly that, with the codes packed on
the device by ``gq_pack_codes`` (each row a little-endian bit stream of
``bits``-wide codes in uint32 words), and ``dequantize`` reproduces the
sweep's dequantized weights bit for bit (``gq_unpack_dequant``).
``save_layer`` / ``load_layer`` write and read one layer's linears, so a
multi-layer run can be resumed layer by layer.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _arrays as A
from . import _lib


@dataclass
class PackedLinear:
    qweight: torch.Tensor   # [m, words] int32 holding the uint32 words
    scales: torch.Tensor    # [m, n // g] float32, permuted group order
    zeros: torch.Tensor     # [m, n // g] float32
    g_idx: torch.Tensor     # [n] int32: group of each original column
    perm: torch.Tensor      # [n] int32: act-order permutation
    bits: int
    group_size: int
    sym: bool
    n: int                  # in_features

    @property
    def m(self) -> int:
        return self.qweight.shape[0]

    def to(self, device) -> "PackedLinear":
        return PackedLinear(self.qweight.to(device), self.scales.to(device), self.zeros.to(device),
                            self.g_idx.to(device), self.perm.to(device), self.bits,
                            self.group_size, self.sym, self.n)


def pack_result(res, bits: int, group_size: int, sym: bool) -> PackedLinear:
    """Pack a sweep / RTN result (``codes``, ``scales``, ``zeros``, ``g_idx``,
    ``perm`` on the device) into a :class:`PackedLinear`."""
    codes = res.codes.contiguous()
    m, n = codes.shape
    words = _lib.lib().gq_packed_words(n, bits)
    if words < 0:
        raise ValueError(f"bits must be 1..8, got {bits}")
    q = torch.empty((m, words), dtype=torch.int32, device=codes.device)
    _lib.call("gq_pack_codes", A.ptr(codes), m, n, n, bits, A.ptr(q), words, A.stream())
    return PackedLinear(q, res.scales.contiguous(), res.zeros.contiguous(),
                        res.g_idx.to(torch.int32).contiguous(), res.perm.to(torch.int32),
                        bits, group_size, bool(sym), n)


def unpack_codes(p: PackedLinear) -> torch.Tensor:
    """uint8 codes [m, n] in original column order."""
    A.require_cuda()
    q = p.qweight.cuda().contiguous()
    out = torch.empty((q.shape[0], p.n), dtype=torch.uint8, device="cuda")
    _lib.call("gq_unpack_dequant", A.ptr(q), q.shape[0], p.n, q.shape[1], p.bits, int(p.sym),
              None, None, 0, None, None, A.ptr(out), A.stream())
    return out


def dequantize(p: PackedLinear) -> torch.Tensor:
    """float32 [m, n]: ``(code + qmin - zero) * scale`` per element."""
    A.require_cuda()
    q = p.qweight.cuda().contiguous()
    s, z, g = (t.cuda().contiguous() for t in (p.scales, p.zeros, p.g_idx))
    out = torch.empty((q.shape[0], p.n), dtype=torch.float32, device="cuda")
    _lib.call("gq_unpack_dequant", A.ptr(q), q.shape[0], p.n, q.shape[1], p.bits, int(p.sym),
              A.ptr(s), A.ptr(z), s.shape[1], A.ptr(g), A.ptr(out), None, A.stream())
    return out


def save_layer(path: str, linears: dict[str, PackedLinear]) -> None:
    """One layer's packed linears to ``path`` (CPU tensors + metadata)."""
    blob = {name: {"qweight": p.qweight.cpu(), "scales": p.scales.cpu(), "zeros": p.zeros.cpu(),
                   "g_idx": p.g_idx.cpu(), "perm": p.perm.cpu(), "bits": p.bits,
                   "group_size": p.group_size, "sym": p.sym, "n": p.n}
            for name, p in linears.items()}
    torch.save({"format": "gq-packed-v1", "linears": blob}, path)


def load_layer(path: str, device: str = "cpu") -> dict[str, PackedLinear]:
    blob = torch.load(path, map_location="cpu", weights_only=True)
    if blob.get("format") != "gq-packed-v1":
        raise ValueError(f"{path}: not a packed layer file")
    return {name: PackedLinear(d["qweight"], d["scales"], d["zeros"], d["g_idx"], d["perm"],
                               int(d["bits"]), int(d["group_size"]), bool(d["sym"]),
                               int(d["n"])).to(device)
            for name, d in blob["linears"].items()}
