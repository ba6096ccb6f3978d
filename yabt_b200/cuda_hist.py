"""Drop-in for the reference's CUDA histogram module (yabt/cuda_hist.py).

Same functions, arguments and result: ``is_available()`` and
``build_hist(binned, slot, g, h, w, K, F, B)`` returning the fused
``(3, K, F, B)`` float32 histogram in which row ``i`` adds
``(g[i], h[i], w[i])`` into bin ``binned[i, f]`` of node slot ``slot[i]`` for
every feature ``f`` (yabt/cuda_hist.py:79-89).

The kernels (``yabt_hist_build`` in libyabt_b200.so) sum exact fixed-point
integers and round each bin once, so the result is deterministic; the
reference's float atomics agree with it to float32 rounding of the sums.
Unlike the reference, bad input is not silently accumulated: a slot outside
``[0, K)``, a bin ``>= B`` or a non-finite value raises ``YabtError`` (the
check reads one device word, which synchronises the stream).
"""

from __future__ import annotations

import torch

from . import _lib

_ERR_BITS = {1 << 4: "slot or bin out of range", 1 << 6: "non-finite g/h/w value"}


def is_available() -> bool:
    """True if the CUDA histogram entry point can run here."""
    try:
        _lib.load()
    except Exception:
        return False
    return torch.cuda.is_available()


def build_hist(binned: torch.Tensor, slot: torch.Tensor, g: torch.Tensor, h: torch.Tensor,
               w: torch.Tensor, K: int, F: int, B: int) -> torch.Tensor:
    """Fused (3, K, F, B) histogram (yabt/cuda_hist.py:79-89). ``binned`` is
    (n, F) uint8 row-major; ``slot`` int64 (n,); ``g/h/w`` float32 (n,)."""
    K, F, B = int(K), int(F), int(B)
    if binned.device.type != "cuda":
        raise ValueError("build_hist needs CUDA tensors")
    if binned.dtype != torch.uint8 or binned.dim() != 2 or binned.shape[1] != F:
        raise ValueError(f"binned must be (n, {F}) uint8, got {tuple(binned.shape)} {binned.dtype}")
    n = binned.shape[0]
    dev = binned.device
    binned = binned.contiguous()
    slot = slot.to(device=dev, dtype=torch.int64).contiguous()
    g = g.to(device=dev, dtype=torch.float32).contiguous()
    h = h.to(device=dev, dtype=torch.float32).contiguous()
    w = w.to(device=dev, dtype=torch.float32).contiguous()
    for name, t in (("slot", slot), ("g", g), ("h", h), ("w", w)):
        if t.shape != (n,):
            raise ValueError(f"{name} must have shape ({n},), got {tuple(t.shape)}")
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(int(lib.yabt_hist_build_workspace_bytes(n, K, F)), dtype=torch.uint8, device=dev)
        out = torch.empty(3, K, F, B, dtype=torch.float32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.check(lib.yabt_hist_build(binned.data_ptr(), slot.data_ptr(), g.data_ptr(), h.data_ptr(),
                                       w.data_ptr(), n, K, F, B, out.data_ptr(), err.data_ptr(),
                                       ws.data_ptr(), ws.numel(), _lib.stream_ptr()), "yabt_hist_build")
        bits = int(err.item())
    if bits:
        why = ", ".join(v for k, v in _ERR_BITS.items() if bits & k) or f"0x{bits:x}"
        raise _lib.YabtError(f"build_hist: {why}")
    return out
