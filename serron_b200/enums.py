"""Enumerations shared by the operators and layers.

Same members and integer encodings as the reference (packages/serron/torch-ext/serron/enums.py:10-53):
the compiled operators take ``border`` and ``algo`` as these integers.
"""

from __future__ import annotations

from enum import Enum, IntEnum


class Operation(Enum):
    """Morphological operations."""

    ERODE = "erode"
    DILATE = "dilate"
    OPEN = "open"
    CLOSE = "close"
    GRADIENT = "gradient"
    TOP_HAT = "top_hat"
    BLACK_HAT = "black_hat"


class BorderMode(Enum):
    """How samples outside the image are formed."""

    REFLECT = "reflect"  #: mirror without repeating the edge sample
    REPLICATE = "replicate"  #: clamp to the edge sample
    CONSTANT = "constant"  #: the neutral element (+inf for erosion, -inf for dilation)


BORDER_TO_INT: dict[BorderMode, int] = {
    BorderMode.REFLECT: 0,
    BorderMode.REPLICATE: 1,
    BorderMode.CONSTANT: 2,
}
"""Integer encoding of :class:`BorderMode` taken by the compiled operators."""


class Algorithm(IntEnum):
    """Algorithm a compiled operator runs; ``AUTO`` lets the library choose, the others force one."""

    AUTO = 0
    ELEMENT = 1
    TILED = 2
    SEPARABLE = 3
