"""Argument contracts of the Python entries, checked before anything is launched.

Every public entry of ``soupsuck_b200.kernels`` states what it accepts as data:
one ``Operand`` rule per tensor argument and ``Number`` / ``Choice`` rules for
the rest.  ``admit(entry, device, name=(value, rule), ...)`` applies them in
order and raises ``ValueError("<entry>: <name> <fault>")`` at the first
violation, so an unsupported call never reaches the C ABI (the drop-in patches
catch exactly this ValueError and run the library's own code instead).  The
rules read tensor metadata only; nothing here synchronises with the device.
"""

from __future__ import annotations

import math
import numbers

import torch

HALF, SINGLE, BYTE, LONG = torch.float16, torch.float32, torch.uint8, torch.int64
FLOATS = (HALF, SINGLE)


def _names(dtypes):
    return "/".join(str(d).replace("torch.", "") for d in dtypes)


class Operand:
    """A tensor operand: dtypes, rank, layout, gradient state and size bounds.

    layout: "dense" (contiguous), "rows" (unit stride in the last dimension only)
    or None (any strides).  ``same_device``: must sit on the entry's device.
    """

    def __init__(self, *dtypes, ndim=None, layout="dense", frozen=False, at_least=0, exactly=None,
                 same_device=True, optional=False):
        self.dtypes = dtypes
        self.ndim = (ndim,) if isinstance(ndim, int) else ndim
        self.layout = layout
        self.frozen = frozen
        self.at_least = at_least
        self.exactly = exactly
        self.same_device = same_device
        self.optional = optional

    def fault(self, value, device):
        if value is None:
            return None if self.optional else "is missing"
        if not isinstance(value, torch.Tensor):
            return f"is a {type(value).__name__}, not a tensor"
        if not value.is_cuda:
            return f"is on {value.device}; the kernels run on CUDA devices only"
        if self.same_device and device is not None and value.device != device:
            return f"is on {value.device} while the call runs on {device}"
        if self.dtypes and value.dtype not in self.dtypes:
            return f"has dtype {_names((value.dtype,))}, accepted: {_names(self.dtypes)}"
        if self.ndim is not None and value.ndim not in self.ndim:
            return f"has {value.ndim} dimensions, accepted: {' or '.join(map(str, self.ndim))}"
        if self.layout == "dense" and not value.is_contiguous():
            return f"is strided {tuple(value.stride())}; a contiguous tensor is required"
        if self.layout == "rows" and value.ndim and value.stride(-1) != 1:
            return "has a strided last dimension; unit stride is required there"
        if self.frozen and value.requires_grad:
            return "requires grad; this operand must be frozen"
        if value.numel() < self.at_least:
            return f"holds {value.numel()} elements, at least {self.at_least} are read"
        if self.exactly is not None and value.numel() != self.exactly:
            return f"holds {value.numel()} elements, exactly {self.exactly} expected"
        return None


class Number:
    """A real scalar; ``finite`` and ``minimum`` bound it, ``integral`` asks for an int."""

    def __init__(self, finite=True, minimum=None, integral=False):
        self.finite, self.minimum, self.integral = finite, minimum, integral

    def fault(self, value, device):
        kind = numbers.Integral if self.integral else numbers.Real
        if isinstance(value, bool) or not isinstance(value, kind):
            return f"is {value!r}; {'an integer' if self.integral else 'a real number'} is required"
        if self.finite and not math.isfinite(value):
            return f"is {value!r}; a finite value is required"
        if self.minimum is not None and value < self.minimum:
            return f"is {value!r}; it may not be below {self.minimum}"
        return None


class Choice:
    """One of a fixed set of values (compared with ``==`` and exact type for bools)."""

    def __init__(self, *allowed):
        self.allowed = allowed

    def fault(self, value, device):
        for option in self.allowed:
            if type(option) is bool or type(value) is bool:
                if value is option:
                    return None
            elif value == option:
                return None
        return f"is {value!r}; accepted: {', '.join(repr(a) for a in self.allowed)}"


def admit(entry, device, /, **checks):
    """Apply each ``name=(value, rule)`` pair in order; raise at the first fault."""
    for name, (value, rule) in checks.items():
        fault = rule.fault(value, device)
        if fault is not None:
            raise ValueError(f"{entry}: {name.replace('__', '.')} {fault}")


def refuse(entry, why):
    raise ValueError(f"{entry}: {why}")
