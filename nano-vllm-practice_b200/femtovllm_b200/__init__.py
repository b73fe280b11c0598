"""femtovllm_b200: B200-native (sm_100a) attention hot path of FemtoVLLM.

Host side of the drop-in boundary.  ``femtovllm_b200._C`` mirrors the
reference's native module ``femtovllm._C`` (same entry points and constants),
``femtovllm_b200.ops`` mirrors ``femtovllm.ops`` (same Python signatures), and
``femtovllm_b200.capi`` binds the raw C ABI of ``libfemtovllm_b200.so`` with
ctypes.  There is no CPU path: importing ``ops`` without the built extension
raises ``ImportError``.
"""

from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "libfemtovllm_b200.so"
EXT_PATH = PACKAGE_DIR / "_C.so"

__all__ = ["PACKAGE_DIR", "LIB_PATH", "EXT_PATH"]
