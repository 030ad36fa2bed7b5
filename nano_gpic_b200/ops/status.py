"""The extension's device error word: kernels that give up a bounded wait record a code there instead of hanging.

Codes (csrc/common.cuh): 1 stage-full wait, 2 stage-empty wait, 3 accumulator-full wait, 4 accumulator-empty wait,
5 drain on unwind, 6 peer flag. `check()` raises NanoCommTimeout / RuntimeError when the word is set.
"""
from .._ext import ext

CODES = {1: "smem stage never filled", 2: "smem stage never freed", 3: "accumulator never ready",
         4: "accumulator never drained", 5: "unwind drain timed out", 6: "peer flag never arrived"}


class NanoCommTimeout(RuntimeError):
    """A device-side bounded wait on peer memory ran out (a peer rank stopped or a message was lost)."""


def read():
    return int(ext().status_read())


def clear():
    ext().status_clear()


class AsyncCheck:
    """The status word checked one step late, without a host synchronisation in the step: `post()` enqueues a copy of
    the word into pinned host memory behind the step's work and records an event; `poll()` (the next step, once that
    event has completed, which it normally has long before) raises as check() does when the copied word is set."""

    def __init__(self):
        import torch
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None

    def post(self):
        import torch
        ext().status_copy_async(self.host)
        self.event = torch.cuda.Event()
        self.event.record()

    def poll(self):
        if self.event is None:
            return
        self.event.synchronize()
        self.event = None
        if int(self.host[0]):
            check()


def check():
    code = read()
    if code:
        clear()
        msg = f"device status word {code}: {CODES.get(code, 'unknown')}"
        raise NanoCommTimeout(msg) if code == 6 else RuntimeError(msg)
