"""GPU test harness that calls the C ABI the way the reference grader does (graders/child.py):

- every pointer argument is a view into a device buffer with 4096 guard bytes (0xA5) on each
  side (child.py:21-23,52-64);
- outputs are filled with 0xFF before each call, inputs are copied in, and after the call the
  guards and the inputs are checked (child.py:141-147,203-204);
- three calls at the same pointers: set A, set B (seed + 7919), set A again, and the third call
  must repeat the first one's bits (child.py:184-207).
"""
import ctypes

import numpy as np
import torch

GUARD = 4096
GUARD_BYTE = 0xA5
POISON = 0xFF
SET_B = 7919


class Guarded:
    def __init__(self, nbytes, dtype, shape, device="cuda", phase=0):
        """`phase` bytes of extra offset make the view deliberately misaligned."""
        self.n = nbytes
        self.phase = phase
        self.raw = torch.full((GUARD + phase + nbytes + GUARD,), GUARD_BYTE, dtype=torch.uint8, device=device)
        self.t = self.raw[GUARD + phase:GUARD + phase + nbytes].view(dtype).view(shape) if nbytes else \
            torch.empty(shape, dtype=dtype, device=device)

    def guards_ok(self):
        lo = self.raw[:GUARD + self.phase]
        hi = self.raw[GUARD + self.phase + self.n:]
        return bool((lo == GUARD_BYTE).all() and (hi == GUARD_BYTE).all())

    def poison(self):
        if self.n:
            self.raw[GUARD + self.phase:GUARD + self.phase + self.n].fill_(POISON)

    def load(self, src):
        if self.n:
            self.t.copy_(src.to(self.t.device).view(self.t.dtype).view(self.t.shape))

    @property
    def ptr(self):
        return ctypes.c_void_p(self.t.data_ptr()) if self.n else ctypes.c_void_p(0)


def nbytes(t):
    return t.numel() * t.element_size()


def guarded_like(t, phase=0):
    return Guarded(nbytes(t), t.dtype, tuple(t.shape), phase=phase)


def as_bytes(t):
    """Raw bytes of a tensor (bit-level comparison, NaN-safe)."""
    return t.detach().cpu().contiguous().reshape(-1).view(torch.uint8)


def _sync(device):
    if torch.device(device).type == "cuda":
        torch.cuda.synchronize()


def protocol_record(call, sets, in_names, out_specs, phase=0, device="cuda"):
    """The grader's 3-call protocol without assertions: per call whether the guards and inputs are
    intact, the outputs (CPU tensors), whether each output element still holds the poison, and
    whether call 3 repeated call 1's bits.  `device` is "cuda" for the kernels and "cpu" for the
    planted-mistake tests, which run the protocol on host buffers."""
    bufs = {k: Guarded(nbytes(sets[0][k]), sets[0][k].dtype, tuple(sets[0][k].shape), device=device, phase=phase)
            for k in in_names}
    for k, (dt, shp) in out_specs.items():
        bufs[k] = Guarded(int(np.prod(shp)) * torch.empty((), dtype=dt).element_size(), dt, tuple(shp),
                          device=device, phase=phase)
    calls = []
    for idx in (0, 1, 0):
        s = sets[idx]
        for k in out_specs:
            bufs[k].poison()
        for k in in_names:
            bufs[k].load(s[k])
        _sync(device)
        call(bufs, s)
        _sync(device)
        rec = {"guards_ok": {k: b.guards_ok() for k, b in bufs.items()},
               "inputs_unchanged": {k: bool(torch.equal(as_bytes(bufs[k].t), as_bytes(s[k]))) for k in in_names},
               "outputs": {k: bufs[k].t.detach().cpu().clone() for k in out_specs}}
        rec["poisoned"] = {k: (as_bytes(v).view(v.numel(), -1) == POISON).all(dim=1) if v.numel() else
                           torch.zeros(0, dtype=torch.bool) for k, v in rec["outputs"].items()}
        calls.append(rec)
    same = all(torch.equal(as_bytes(calls[0]["outputs"][k]), as_bytes(calls[2]["outputs"][k])) for k in out_specs)
    return {"calls": calls, "identical_repeat": same}


def case_label(record, bad_call1, bad_call2):
    """The grader's verdict for one case (graders/verdict.py:34-61): None when it passes, else the
    label of the first failed check.  bad_callN = {output name: boolean mask of elements outside
    the tolerance of the oracle on that call's inputs}."""
    for c in record["calls"]:
        if not all(c["guards_ok"].values()):
            return "out-of-bounds write"
        if not all(c["inputs_unchanged"].values()):
            return "input modified"
    for name, bad in bad_call1.items():
        if bool(bad.any()):
            poisoned = record["calls"][0]["poisoned"][name].reshape(-1)
            if bool((poisoned | ~bad.reshape(-1)).all()):
                return "unwritten output"
            return "wrong value"
    for name, bad in bad_call2.items():
        if bool(bad.any()):
            return "stale state"
    return None


def three_call(call, sets, in_names, out_specs, phase=0):
    """Run the grader's 3-call protocol.

    call(bufs) issues the C-ABI call with pointers from `bufs` (name -> Guarded) and the scalars of
    the current set; sets = [set_a, set_b] input dicts (CPU tensors + scalars); out_specs =
    {name: (dtype, shape)}.  Returns ([outputs of call 1, call 2], identical_repeat) with CPU
    tensors, after asserting guards and input integrity on every call."""
    rec = protocol_record(call, sets, in_names, out_specs, phase=phase)
    for c in rec["calls"]:
        for k, ok in c["guards_ok"].items():
            assert ok, f"guard bytes around {k} were overwritten"
        for k, ok in c["inputs_unchanged"].items():
            assert ok, f"input {k} was modified"
    return [rec["calls"][0]["outputs"], rec["calls"][1]["outputs"]], rec["identical_repeat"]
