"""HPC domain: linear extrapolation predictor and error-bounded INT16
codecs with RLE / BlockSparse / BlockSparse+RLE packing (nangila-hpc)."""
from .linear import LinearPredictor
from .quantizers import (BlockSparseQuantizer, BlockSparseRleQuantizer, ErrorBoundedQuantizer, QuantizerError,
                         RunLengthQuantizer, rle_decode_i16, rle_encode_i16)

__all__ = [
    "LinearPredictor", "BlockSparseQuantizer", "BlockSparseRleQuantizer", "ErrorBoundedQuantizer",
    "QuantizerError", "RunLengthQuantizer", "rle_decode_i16", "rle_encode_i16",
]
