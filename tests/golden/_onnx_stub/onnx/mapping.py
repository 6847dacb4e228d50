"""Inert submodule of the onnx stand-in (see the package docstring)."""


def __getattr__(name):
    from . import _Inert
    return _Inert()
