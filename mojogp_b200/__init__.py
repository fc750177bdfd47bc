"""mojogp_b200 — B200-native exact-GP hot path (matrix-free K·V, mBCG, pivoted
Cholesky, LOVE) behind MojoGP's SingleOutputGP / MultiOutputLMCGP surface."""
from .kernel import (RBF, RQ, Kernel, KernelNode, KernelType, Linear, Matern12, Matern32,
                     Matern52, Periodic, Polynomial, make_ard_kernel)

__version__ = "0.1.0"
