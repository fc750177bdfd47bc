"""mojogp_b200 — B200-native exact-GP hot path (matrix-free K·V, mBCG, pivoted
Cholesky, LOVE) behind MojoGP's SingleOutputGP / MultiOutputLMCGP surface."""
from .gp import PredictionResult, SingleOutputGP, TrainingResult, fit_gp
from .kernel import (RBF, RQ, Kernel, KernelNode, KernelType, Linear, Matern12, Matern32,
                     Matern52, Periodic, Polynomial, make_ard_kernel)
from .multi_output_gp import MultiOutputGP, MultiOutputLMCGP, MultiOutputPredictionResult
from .utils import StandardScaler

# The reference's top-level names (mojogp/__init__.py) for the routes built here.
__all__ = ["SingleOutputGP", "fit_gp", "StandardScaler", "MultiOutputGP", "MultiOutputPredictionResult", "MultiOutputLMCGP", "TrainingResult",
           "PredictionResult", "Kernel", "KernelNode", "KernelType", "RBF", "RQ", "Linear",
           "Matern12", "Matern32", "Matern52", "Periodic", "Polynomial", "make_ard_kernel"]

__version__ = "0.1.0"
