"""Kernel objects: the public kernel-tree surface and its device encoding.

Mirrors the continuous part of the reference's kernel API
(mojogp/kernel.py:21-70 KernelType, 177-720 KernelNode, 1247-1520 Kernel
factories, 1520-1600 make_ard_kernel): the same constructors, composition
operators (+, *, scalar *), active_dims, ARD resolution, parameter names,
parameter counts and public parameter order.

Instead of the reference's SymPy -> Mojo codegen
(mojogp/codegen_engine/expressions.py:424-650), a tree is encoded as the flat
int32 post-order program declared in include/gpb200.h and evaluated by the
CUDA library. The engine parameter layout equals the public layout returned
by get_param_names(); a scale node's parameter follows its child's
parameters (kernel.py:553-556).
"""
from __future__ import annotations

import copy
from dataclasses import dataclass
from enum import Enum
from typing import Dict, List, Optional, Sequence, Union

import numpy as np

GPB_SPEC_VERSION = 1
NODE_LEAF, NODE_SUM, NODE_PRODUCT, NODE_SCALE = 1, 2, 3, 4


class KernelType(Enum):
    """Continuous kernel families (reference kernel.py:21-40)."""

    RBF = 0
    MATERN12 = 1
    MATERN32 = 2
    MATERN52 = 3
    RQ = 4
    PERIODIC = 5
    LINEAR = 6
    POLYNOMIAL = 7


@dataclass
class KernelNode:
    """A node in the kernel composition tree (reference kernel.py:177-200)."""

    kernel_type: Optional[KernelType] = None
    operator: Optional[str] = None  # "sum", "product", "scale"
    left: Optional["KernelNode"] = None
    right: Optional["KernelNode"] = None
    scale_factor: Optional[float] = None
    ard_dim: Optional[int] = None
    initial_values: Optional[Dict[str, float]] = None
    ard: bool = False
    active_dims: Optional[tuple] = None

    # ------------------------------------------------------------ composition
    def __add__(self, other: "KernelNode") -> "KernelNode":
        return KernelNode(operator="sum", left=self, right=other)

    def __radd__(self, other):
        if isinstance(other, (int, float)) and other == 0:
            return self
        return KernelNode(operator="sum", left=other, right=self)

    def __mul__(self, other: Union["KernelNode", float, int]) -> "KernelNode":
        if isinstance(other, (float, int)):
            return KernelNode(operator="scale", left=self, scale_factor=float(other))
        return KernelNode(operator="product", left=self, right=other)

    def __rmul__(self, other):
        if isinstance(other, (float, int)):
            return KernelNode(operator="scale", left=self, scale_factor=float(other))
        return KernelNode(operator="product", left=other, right=self)

    def with_active_dims(self, dims: Sequence[int]) -> "KernelNode":
        """Restrict this (possibly composite) kernel to the given input dims."""
        new_node = copy.deepcopy(self)
        new_node.active_dims = tuple(sorted(int(d) for d in dims))
        return new_node

    # --------------------------------------------------------------- queries
    def is_leaf(self) -> bool:
        return self.kernel_type is not None

    def has_ard(self) -> bool:
        if self.is_leaf():
            return bool(self.ard) or self.ard_dim is not None
        return (self.left is not None and self.left.has_ard()) or (
            self.right is not None and self.right.has_ard()
        )

    def num_params(self) -> int:
        """Parameter count (reference kernel.py:324-365)."""
        if self.is_leaf():
            kt = self.kernel_type
            if self.ard_dim is not None:
                if kt in (KernelType.PERIODIC, KernelType.RQ):
                    return self.ard_dim + 2
                if kt == KernelType.POLYNOMIAL:
                    return self.ard_dim + 3
                return self.ard_dim + 1
            if kt == KernelType.POLYNOMIAL:
                return 3
            if kt in (KernelType.PERIODIC, KernelType.RQ):
                return 3
            return 2
        if self.operator in ("sum", "product"):
            return self.left.num_params() + self.right.num_params()
        if self.operator == "scale":
            return self.left.num_params() + 1
        raise ValueError(f"Unknown operator: {self.operator}")

    def get_param_names(self, prefix: str = "") -> List[str]:
        """Parameter names in public order (reference kernel.py:367-449)."""
        if self.is_leaf():
            base = self.kernel_type.name.lower()
            if prefix:
                base = f"{prefix}_{base}"
            kt = self.kernel_type
            if self.ard_dim is not None:
                names = [f"{base}_ls_{d}" for d in range(self.ard_dim)]
                if kt == KernelType.PERIODIC:
                    names.append(f"{base}_period")
                elif kt == KernelType.RQ:
                    names.append(f"{base}_alpha")
                elif kt == KernelType.POLYNOMIAL:
                    names += [f"{base}_degree", f"{base}_offset"]
                names.append(f"{base}_outputscale")
                return names
            if kt == KernelType.POLYNOMIAL:
                return [f"{base}_degree", f"{base}_offset", f"{base}_outputscale"]
            if kt == KernelType.LINEAR:
                return [f"{base}_variance", f"{base}_outputscale"]
            if kt in (KernelType.PERIODIC, KernelType.RQ):
                extra = "period" if kt == KernelType.PERIODIC else "alpha"
                return [f"{base}_lengthscale", f"{base}_{extra}", f"{base}_outputscale"]
            return [f"{base}_lengthscale", f"{base}_outputscale"]
        if self.operator in ("sum", "product"):
            lp = f"{prefix}left" if prefix else "left"
            rp = f"{prefix}right" if prefix else "right"
            return self.left.get_param_names(lp) + self.right.get_param_names(rp)
        if self.operator == "scale":
            return self.left.get_param_names(prefix) + [f"{prefix}_scale" if prefix else "scale"]
        raise ValueError(f"Unknown operator: {self.operator}")

    def get_initial_params(self) -> np.ndarray:
        """Initial values (defaults 1.0) in public order (kernel.py:451-460, 631-666)."""
        values = np.ones(self.num_params(), dtype=np.float32)
        self._fill_initial_params(values, 0)
        return values

    def _fill_initial_params(self, values: np.ndarray, offset: int) -> int:
        if self.is_leaf():
            n = self.num_params()
            if self.initial_values:
                for i, name in enumerate(self.get_param_names()):
                    for key, val in self.initial_values.items():
                        if name.endswith(f"_{key}") or name == key:
                            values[offset + i] = val
                            break
            return offset + n
        if self.operator in ("sum", "product"):
            mid = self.left._fill_initial_params(values, offset)
            return self.right._fill_initial_params(values, mid)
        if self.operator == "scale":
            mid = self.left._fill_initial_params(values, offset)
            if self.initial_values and "scale" in self.initial_values:
                values[mid] = self.initial_values["scale"]
            elif self.scale_factor is not None:
                values[mid] = self.scale_factor
            return mid + 1
        return offset

    def engine_num_params(self) -> int:
        return self.num_params()

    def engine_trainable_mask(self) -> np.ndarray:
        """Which parameters Adam may move: a polynomial degree stays fixed."""
        mask = np.ones(self.num_params(), dtype=np.bool_)
        self._fill_trainable(mask, 0)
        return mask

    def _fill_trainable(self, mask: np.ndarray, offset: int) -> int:
        if self.is_leaf():
            if self.kernel_type == KernelType.POLYNOMIAL:
                nd = self.ard_dim or 0
                mask[offset + nd] = False
            return offset + self.num_params()
        if self.operator in ("sum", "product"):
            return self.right._fill_trainable(mask, self.left._fill_trainable(mask, offset))
        return self.left._fill_trainable(mask, offset) + 1

    def to_engine_params(self, public_params: np.ndarray) -> np.ndarray:
        p = np.asarray(public_params, dtype=np.float32)
        if p.shape != (self.num_params(),):
            raise ValueError(
                f"public_params must have shape ({self.num_params()},), got {p.shape}"
            )
        return p.copy()

    def from_engine_params(self, engine_params: np.ndarray) -> np.ndarray:
        return self.to_engine_params(engine_params)

    # -------------------------------------------------------------- encoding
    def to_spec(self, dim: int) -> np.ndarray:
        """Encode the tree as the int32 post-order program of gpb200.h."""
        words: List[int] = []
        nodes = [0]

        def leaf_dims(node: "KernelNode", inherited: Optional[tuple]) -> List[int]:
            dims = node.active_dims if node.active_dims is not None else inherited
            if dims is None:
                return list(range(dim))
            return [int(d) for d in dims]

        def emit(node: "KernelNode", offset: int, inherited: Optional[tuple]) -> int:
            dims_here = node.active_dims if node.active_dims is not None else inherited
            if node.is_leaf():
                dl = leaf_dims(node, inherited)
                for d in dl:
                    if not 0 <= d < dim:
                        raise ValueError(f"active dim {d} out of range for input dim {dim}")
                ard = node.ard_dim is not None or bool(node.ard)
                if ard and node.ard_dim is not None and node.ard_dim != len(dl):
                    raise ValueError(
                        f"ARD kernel has {node.ard_dim} lengthscales but {len(dl)} active dims"
                    )
                words.extend([NODE_LEAF, node.kernel_type.value, int(ard), offset, len(dl)] + dl)
                nodes[0] += 1
                return offset + node.num_params()
            if node.operator in ("sum", "product"):
                mid = emit(node.left, offset, dims_here)
                end = emit(node.right, mid, dims_here)
                words.append(NODE_SUM if node.operator == "sum" else NODE_PRODUCT)
                nodes[0] += 1
                return end
            if node.operator == "scale":
                mid = emit(node.left, offset, dims_here)
                words.extend([NODE_SCALE, mid])
                nodes[0] += 1
                return mid + 1
            raise ValueError(f"Unknown operator: {node.operator}")

        resolved = self.resolve_ard(dim)
        total = emit(resolved, 0, None)
        if total != resolved.num_params():
            raise AssertionError("parameter layout mismatch")
        return np.asarray([GPB_SPEC_VERSION, total, nodes[0]] + words, dtype=np.int32)

    def resolve_ard(self, dim: int) -> "KernelNode":
        """Give every leaf that asked for ARD its lengthscale count."""
        if self.is_leaf():
            node = copy.copy(self)
            if self.ard and self.ard_dim is None:
                node.ard_dim = len(self.active_dims) if self.active_dims is not None else dim
            return node
        node = copy.copy(self)
        node.left = self.left.resolve_ard(dim) if self.left is not None else None
        node.right = self.right.resolve_ard(dim) if self.right is not None else None
        return node

    def to_dict(self) -> dict:
        d: dict = {}
        if self.is_leaf():
            d["kernel_type"] = self.kernel_type.name
            if self.ard:
                d["ard"] = True
            if self.ard_dim is not None:
                d["ard_dim"] = int(self.ard_dim)
            if self.initial_values:
                d["initial_values"] = {k: float(v) for k, v in self.initial_values.items()}
        else:
            d["operator"] = self.operator
            d["left"] = self.left.to_dict()
            if self.right is not None:
                d["right"] = self.right.to_dict()
            if self.scale_factor is not None:
                d["scale_factor"] = float(self.scale_factor)
        if self.active_dims is not None:
            d["active_dims"] = list(self.active_dims)
        return d

    @staticmethod
    def from_dict(d: dict) -> "KernelNode":
        if "kernel_type" in d:
            return KernelNode(
                kernel_type=KernelType[d["kernel_type"]],
                ard=d.get("ard", False),
                ard_dim=d.get("ard_dim"),
                initial_values=d.get("initial_values"),
                active_dims=tuple(d["active_dims"]) if d.get("active_dims") is not None else None,
            )
        return KernelNode(
            operator=d["operator"],
            left=KernelNode.from_dict(d["left"]),
            right=KernelNode.from_dict(d["right"]) if "right" in d else None,
            scale_factor=d.get("scale_factor"),
            active_dims=tuple(d["active_dims"]) if d.get("active_dims") is not None else None,
        )

    def __repr__(self) -> str:
        if self.is_leaf():
            name = {
                KernelType.RBF: "RBF",
                KernelType.MATERN12: "Matern12",
                KernelType.MATERN32: "Matern32",
                KernelType.MATERN52: "Matern52",
                KernelType.RQ: "RQ",
                KernelType.PERIODIC: "Periodic",
                KernelType.LINEAR: "Linear",
                KernelType.POLYNOMIAL: "Polynomial",
            }[self.kernel_type]
            extra = []
            if self.ard:
                extra.append("ard=True")
            if self.active_dims is not None:
                extra.append(f"active_dims={list(self.active_dims)}")
            return f"{name}({', '.join(extra)})"
        if self.operator == "sum":
            return f"({self.left!r} + {self.right!r})"
        if self.operator == "product":
            return f"({self.left!r} * {self.right!r})"
        return f"{self.scale_factor} * {self.left!r}"


def _leaf(kt: KernelType, ard: bool, active_dims, **init) -> KernelNode:
    return KernelNode(
        kernel_type=kt,
        ard=ard,
        initial_values=init,
        active_dims=tuple(sorted(active_dims)) if active_dims is not None else None,
    )


class Kernel:
    """Kernel factories (reference kernel.py:1247-1432)."""

    @staticmethod
    def rbf(lengthscale: float = 1.0, outputscale: float = 1.0, ard: bool = False,
            active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.RBF, ard, active_dims, lengthscale=lengthscale,
                     outputscale=outputscale)

    @staticmethod
    def matern12(lengthscale: float = 1.0, outputscale: float = 1.0, ard: bool = False,
                 active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.MATERN12, ard, active_dims, lengthscale=lengthscale,
                     outputscale=outputscale)

    @staticmethod
    def matern32(lengthscale: float = 1.0, outputscale: float = 1.0, ard: bool = False,
                 active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.MATERN32, ard, active_dims, lengthscale=lengthscale,
                     outputscale=outputscale)

    @staticmethod
    def matern52(lengthscale: float = 1.0, outputscale: float = 1.0, ard: bool = False,
                 active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.MATERN52, ard, active_dims, lengthscale=lengthscale,
                     outputscale=outputscale)

    @staticmethod
    def periodic(lengthscale: float = 1.0, period: float = 1.0, outputscale: float = 1.0,
                 ard: bool = False, active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.PERIODIC, ard, active_dims, lengthscale=lengthscale,
                     period=period, outputscale=outputscale)

    @staticmethod
    def linear(variance: float = 1.0, outputscale: float = 1.0, ard: bool = False,
               active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.LINEAR, ard, active_dims, variance=variance,
                     outputscale=outputscale)

    @staticmethod
    def rq(lengthscale: float = 1.0, alpha: float = 1.0, outputscale: float = 1.0,
           ard: bool = False, active_dims: Optional[List[int]] = None) -> KernelNode:
        return _leaf(KernelType.RQ, ard, active_dims, lengthscale=lengthscale, alpha=alpha,
                     outputscale=outputscale)

    @staticmethod
    def polynomial(degree: float = 2.0, offset: float = 1.0, outputscale: float = 1.0,
                   active_dims: Optional[List[int]] = None) -> KernelNode:
        d = float(degree)
        if abs(d - round(d)) > 1e-5 or round(d) < 1:
            raise ValueError(f"Polynomial kernel degree must be a positive integer, got {degree}")
        return _leaf(KernelType.POLYNOMIAL, False, active_dims, degree=d, offset=offset,
                     outputscale=outputscale)


def make_ard_kernel(kernel: KernelNode, dim: int) -> KernelNode:
    """Give every continuous leaf per-dimension lengthscales (kernel.py:1520-1583)."""
    if kernel.is_leaf():
        ard_dim = len(kernel.active_dims) if kernel.active_dims is not None else dim
        return KernelNode(
            kernel_type=kernel.kernel_type,
            ard_dim=ard_dim,
            initial_values=kernel.initial_values,
            ard=kernel.ard,
            active_dims=kernel.active_dims,
        )
    return KernelNode(
        operator=kernel.operator,
        left=make_ard_kernel(kernel.left, dim),
        right=make_ard_kernel(kernel.right, dim) if kernel.right is not None else None,
        scale_factor=kernel.scale_factor,
        active_dims=kernel.active_dims,
    )


RBF = Kernel.rbf
Matern12 = Kernel.matern12
Matern32 = Kernel.matern32
Matern52 = Kernel.matern52
Periodic = Kernel.periodic
Linear = Kernel.linear
RQ = Kernel.rq
Polynomial = Kernel.polynomial
