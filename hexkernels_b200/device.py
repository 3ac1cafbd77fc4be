"""Device-pointer launchers over libhexcuda (asynchronous, inputs resident in
HBM).  Arguments may be torch CUDA tensors (their data_ptr() is passed) or raw
integer device addresses; scalars pass through.  ``bind_stream`` makes the
launches go to torch's current stream so torch.cuda.Event timing brackets them.
"""
from __future__ import annotations

from ._lib import check, load


def _arg(a):
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a


def launch(name: str, dev: int, *args) -> None:
    """Call ``hexcuda_<name>(dev, *args)``; raises on a non-zero status."""
    fn = getattr(load(), "hexcuda_" + name)
    check(fn(dev, *[_arg(a) for a in args]))


def bind_stream(dev: int, stream=None) -> None:
    """Route device `dev`'s launches to a torch stream (default: current)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    check(load().hexcuda_set_stream(dev, s.cuda_stream))


def sync(dev: int = -1) -> None:
    check(load().hexcuda_sync(dev))


def launch_count() -> int:
    return int(load().hexcuda_launch_count())
