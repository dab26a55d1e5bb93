"""Class composition for the impl swap (``impl.__class__ = composed``).

A live vLLM impl can only change its class to one with the same instance
layout.  A class built as ``(Mixin, Base)`` gets the mixin as its layout base,
which CPython rejects for the assignment (vLLM-CUDA's impls carry their
``__dict__`` through an ``abc.ABC`` / ``Generic`` base).  ``compose`` builds a
plain single-inheritance subclass of ``Base`` instead, with the mixin's
attributes copied in front of the base's and the mixin registered as its
virtual base (``isinstance(impl, Mixin)`` holds); ``cls._oscar_base`` names
the wrapped class for calls through to it.
"""
from __future__ import annotations

_SKIP = {"__dict__", "__weakref__", "__module__", "__doc__", "__abstractmethods__", "_abc_impl", "__slots__",
         "__qualname__"}


def compose(mixin: type, base: type, name: str, module: str) -> type:
    ns = {k: v for k, v in vars(mixin).items() if k not in _SKIP}
    ns["__module__"] = module
    ns["__doc__"] = f"{base.__name__} with the methods of {mixin.__name__} in front."
    ns["_oscar_base"] = base
    cls = type(name, (base,), ns)
    mixin.register(cls)
    return cls
