"""Inert stand-in for the ``onnx`` package (not installed in this container).

It exists only so that the reference simulator's numeric modules import when
the golden-vector generator (tests/golden/make_golden.py) runs here.  Nothing
in it parses or builds ONNX models: graphs are built from node descriptors.
"""


class _Inert:
    def __init__(self, *args, **kwargs):
        self.args, self.kwargs = args, kwargs

    def __getattr__(self, name):
        return _Inert()

    def __call__(self, *args, **kwargs):
        return _Inert()


class TensorProto:
    UNDEFINED, FLOAT, UINT8, INT8, UINT16, INT16, INT32, INT64 = 0, 1, 2, 3, 4, 5, 6, 7
    STRING, BOOL, FLOAT16, DOUBLE, UINT32, UINT64 = 8, 9, 10, 11, 12, 13
    COMPLEX64, COMPLEX128, BFLOAT16 = 14, 15, 16


class AttributeProto:
    UNDEFINED, FLOAT, INT, STRING, TENSOR, GRAPH = 0, 1, 2, 3, 4, 5
    FLOATS, INTS, STRINGS, TENSORS, GRAPHS = 6, 7, 8, 9, 10


class NodeProto(_Inert):
    pass


class ModelProto(_Inert):
    pass


class GraphProto(_Inert):
    pass


class ValueInfoProto(_Inert):
    pass


class TypeProto(_Inert):
    pass


def load(*args, **kwargs):
    raise RuntimeError("onnx stub: model loading is not available")


def __getattr__(name):
    return _Inert
