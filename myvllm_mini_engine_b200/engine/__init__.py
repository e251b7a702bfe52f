from .batch import PrefillBatch

__all__ = ["PrefillBatch"]
