"""Drop-in replacement of the reference's ``src.model`` package (same public names)."""
from .chassis import KVCache, WalshConfig
from .mhc import SinkhornKnopp, mHCResidualStream, mHCWalsh

__all__ = ["WalshConfig", "KVCache", "mHCWalsh", "mHCResidualStream", "SinkhornKnopp"]
