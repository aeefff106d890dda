"""fusionpass_b200: sm_100a (B200) backend for the fused steps of fusionpass plans.

Public API mirrors the reference package ``fusionpass``: ``execute_plan``,
``validate_plan``, ``verify_equivalence`` / ``assert_equivalent``, ``benchmark``;
fused steps run in ``libfpkern.so`` (C ABI in ``include/fpkern.h``).
"""

from .api import CompiledModel, compile_model
from .bench import BenchResult, UnverifiedSpeedupError, benchmark
from .kernels import DescriptorWriter, KernelTable, launch_step, load_kernels
from .planner import UnsupportedOp
from .runtime import execute_plan
from .validate import validate_plan
from .verify import EquivalenceError, VerifyReport, assert_equivalent, verify_equivalence

__all__ = [
    "compile_model",
    "CompiledModel",
    "UnsupportedOp",
    "execute_plan",
    "validate_plan",
    "launch_step",
    "load_kernels",
    "DescriptorWriter",
    "KernelTable",
    "verify_equivalence",
    "assert_equivalent",
    "EquivalenceError",
    "VerifyReport",
    "benchmark",
    "BenchResult",
    "UnverifiedSpeedupError",
]
