"""The gemm/ tuner's interface rebuilt for q4b_gemm_f16: problems and their files (shapes), the CUDA
schedule space (schedule), legality (verifier), ranking (cost_model), the harness driver (harness),
the search (search) and the correctness fuzz (fuzz)."""

from .schedule import Schedule, default_schedule
from .shapes import BY_ID, EXTRA, REF_SHAPES, SHAPES, TOL, Shape, make_data, read_meta
from .verifier import Verdict, library_accepts, verify

__all__ = ["Shape", "SHAPES", "EXTRA", "REF_SHAPES", "BY_ID", "TOL", "make_data", "read_meta", "Schedule",
           "default_schedule", "verify", "Verdict", "library_accepts"]
