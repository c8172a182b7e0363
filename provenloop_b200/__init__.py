"""provenloop_b200 -- B200-native (sm_100a) CKKS engine for TenSafe's
encrypted LoRA-delta hot path.

* ``provenloop_b200.tensafe_he``: drop-in for the PyO3 module ``tensafe_he``.
* ``provenloop_b200.backend``: engine adapter, ZeRo-MOAI deltas, DP noise.
* ``include/tsgpu.h`` / ``libtsgpu.so``: the C ABI underneath.
"""
__version__ = "0.1.0"
