"""Named implementations of one op family, each declaring where it can run.

Inside vinfer this module is vinfer's own kernel registry: ``BackendRegistry`` and
``BackendContext`` are imported from ``vinfer.kernels.registry`` (``src/vinfer/kernels/
registry.py:25-88``), so the ``sampler`` family and its backends register in the engine's
registry itself. Where vinfer is not installed (a bare GPU host running this package's tests and
benchmarks) the same contract is provided below: a family has one registry; a backend is a
class registered under a name with the device types and dtypes it supports plus an optional
``supports(ctx)`` predicate that returns the reason it cannot run; it is constructed once as
``cls(BackendContext(device, dtype))`` and may set up per-device workspaces then. Choosing a
backend that cannot run fails at resolution with a ``ValueError`` naming the reason; nothing
ever falls back to another backend. ``SOURCE`` says which one is in use.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Generic, TypeVar

import torch

T = TypeVar("T")

try:  # the engine's own registry, when this package runs inside vinfer
    from vinfer.kernels.registry import BackendContext, BackendRegistry  # noqa: F401

    SOURCE = "vinfer"
except ImportError:
    SOURCE = "local"

if SOURCE == "local":

    @dataclass(frozen=True)
    class BackendContext:
        device: torch.device
        dtype: torch.dtype


    @dataclass(frozen=True)
    class _Registration(Generic[T]):
        factory: Callable[[BackendContext], T]
        devices: frozenset[str] | None
        dtypes: frozenset[torch.dtype] | None
        supports: Callable[[BackendContext], str | None] | None

        def why_not(self, ctx: BackendContext) -> str | None:
            if self.devices is not None and ctx.device.type not in self.devices:
                return f"does not run on {ctx.device.type} (supports {sorted(self.devices)})"
            if self.dtypes is not None and ctx.dtype not in self.dtypes:
                return f"does not support {ctx.dtype} (supports {sorted(map(str, self.dtypes))})"
            return None if self.supports is None else self.supports(ctx)


    class BackendRegistry(Generic[T]):
        """Registry of one op family (``sampler`` here)."""

        def __init__(self, family: str) -> None:
            self.family = family
            self._by_name: dict[str, _Registration[T]] = {}

        def register(
            self,
            name: str,
            *,
            devices: set[str] | None = None,
            dtypes: set[torch.dtype] | None = None,
            supports: Callable[[BackendContext], str | None] | None = None,
        ) -> Callable[[Callable[[BackendContext], T]], Callable[[BackendContext], T]]:
            """Class decorator registering ``cls`` under ``name``; a name registers once."""

            def decorate(factory: Callable[[BackendContext], T]) -> Callable[[BackendContext], T]:
                if name in self._by_name:
                    raise ValueError(f"{self.family} backend {name!r} registered twice")
                self._by_name[name] = _Registration(
                    factory,
                    None if devices is None else frozenset(devices),
                    None if dtypes is None else frozenset(dtypes),
                    supports,
                )
                return factory

            return decorate

        def names(self) -> list[str]:
            return sorted(self._by_name)

        def unsupported(self, name: str, ctx: BackendContext) -> str | None:
            """Why ``name`` cannot run in ``ctx``, or ``None`` if it can."""
            reg = self._by_name.get(name)
            if reg is None:
                return f"unknown {self.family} backend {name!r}; available: {self.names()}"
            return reg.why_not(ctx)

        def resolve(self, name: str, ctx: BackendContext) -> T:
            reason = self.unsupported(name, ctx)
            if reason is not None:
                known = name in self._by_name
                raise ValueError((f"{self.family} backend {name!r} " if known else "") + reason)
            return self._by_name[name].factory(ctx)
