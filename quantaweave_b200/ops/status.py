"""Device status words -> host exceptions.

Every bounded wait in the native kernels (mbarrier phases, TMEM hand-offs, peer flags) gives up after its time budget,
records a code in its file's device status word and returns, so a lost signal never hangs the GPU
(``csrc/common.cuh``). ``check_device_status`` reads and clears those words (a device synchronisation) and raises:
``CommTimeoutError`` when a peer's flag never arrived (a dead, stalled or diverged rank), ``DeviceStatusError``
otherwise. The trainer calls it at every logging step, ``bench.py`` after the timed steps.
"""

from __future__ import annotations

STATUS_MESSAGES = {
    1: "a tensor-core pipeline waited too long for a TMA stage",
    2: "a TMA producer waited too long for a free stage",
    3: "an epilogue waited too long for its accumulator",
    4: "an MMA issuer waited too long for the epilogue to release TMEM",
    5: "a peer rank's flag never arrived (a dead, stalled or diverged rank)",
    6: "a debug bounds check failed (QW_DEBUG_BOUNDS build)",
}
PEER_TIMEOUT = 5


class DeviceStatusError(RuntimeError):
    def __init__(self, code: int) -> None:
        self.code = code
        super().__init__(f"device status {code}: {STATUS_MESSAGES.get(code, 'unknown error code')}")


class CommTimeoutError(DeviceStatusError):
    """A device-side wait on another rank timed out."""


def check_device_status(clear: bool = True) -> None:
    """Raise if any native kernel recorded an error since the last check (no-op without the extension)."""
    from . import _load

    C = _load()
    if C is None:
        return
    code = int(C.read_status(clear))
    if code == PEER_TIMEOUT:
        raise CommTimeoutError(code)
    if code:
        raise DeviceStatusError(code)
