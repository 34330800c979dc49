"""mlx.nn stand-in: the activations the MoE block uses."""
from . import core as _mx


def silu(x):
    """x * sigmoid(x); for half-precision inputs the sigmoid is rounded to
    the input dtype before the product, which is rounded again."""
    return x * _mx.sigmoid(x)


def sigmoid(x):
    return _mx.sigmoid(x)
