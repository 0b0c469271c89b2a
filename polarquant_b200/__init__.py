"""polarquant_b200: B200-native (sm_100a) drop-in for the encode and ADC-search
path of the `remex` package (oaustegard/polarquant).

Exports the same names as remex/__init__.py; the corpus lives on the GPU and
every step of encode and search runs as a CUDA kernel of this package's
library (include/polarquant_b200.h).
"""

import warnings

from .core import CompressedVectors, PackedVectors, Quantizer
from .ivf import IVFCoarseIndex
from .packing import pack, packed_nbytes, unpack
from .params import lloyd_max_codebook, nested_codebooks
from .pq_format import load_pq, save_params, save_pq

__version__ = "0.5.0"
__all__ = [
    "Quantizer", "CompressedVectors", "PackedVectors",
    "PolarQuantizer",
    "IVFCoarseIndex",
    "lloyd_max_codebook", "nested_codebooks",
    "pack", "unpack", "packed_nbytes",
    "save_pq", "load_pq", "save_params",
]


def __getattr__(name):
    if name == "PolarQuantizer":
        warnings.warn(
            "PolarQuantizer has been renamed to Quantizer. "
            "The PolarQuantizer alias is deprecated and will be "
            "removed in a future release.",
            DeprecationWarning,
            stacklevel=2,
        )
        return Quantizer
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
