// Kernel-tree program: host parser for the flat int32 spec (gpb200.h) and the
// device-side evaluator used by the generic (composite) tiles and by the
// per-pair gradient code.
//
// Formulas follow the post-pass expressions the reference codegen emits
// (mojogp/codegen_engine/expressions.py:77-420 after
// codegen_engine/passes/numerical_stability.py:13-112). Which exponentials
// carry the max(arg, -20) clamp was read from the generated forward kernels:
// Matern-1/2 ARD, Matern-3/2 and Matern-5/2 (iso and ARD) are clamped; RBF,
// Matern-1/2 isotropic, RQ and Periodic are not. Periodic uses sin^2 / l (not
// l^2) as in expressions.py:240-284. Polynomial carries a fixed integer degree
// (expressions.py:57-73).
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

#include "gpb200.h"
#include "gpb_common.cuh"

namespace gpb {

struct LeafDesc {
  int32_t type;
  int32_t ard;
  int32_t pofs;   // first parameter index of this leaf
  int32_t ndims;  // number of active dims
  int32_t dims[GPB_MAX_DIM];
};

// Post-order program. node_op: GPB_NODE_*; node_arg: leaf index for leaves,
// parameter index for scale nodes.
struct DevKernel {
  int32_t nparams;
  int32_t nnodes;
  int32_t nleaves;
  int32_t d;
  int32_t node_op[GPB_MAX_NODES];
  int32_t node_arg[GPB_MAX_NODES];
  LeafDesc leaf[GPB_MAX_LEAVES];
  float params[GPB_MAX_PARAMS];
};

__host__ __device__ inline int leaf_num_params(int type, int ard, int ndims) {
  switch (type) {
    case GPB_KERNEL_RBF:
    case GPB_KERNEL_MATERN12:
    case GPB_KERNEL_MATERN32:
    case GPB_KERNEL_MATERN52:
      return (ard ? ndims : 1) + 1;
    case GPB_KERNEL_RQ:
    case GPB_KERNEL_PERIODIC:
      return (ard ? ndims : 1) + 2;
    case GPB_KERNEL_LINEAR:
      return (ard ? ndims : 1) + 1;
    case GPB_KERNEL_POLYNOMIAL:
      return ard ? ndims + 3 : 3;
    default:
      return -1;
  }
}

// Parses and validates a spec; fills `k` (params left zero). Returns GPB_OK or
// GPB_ERR_INVALID with a message.
int parse_spec(const int32_t* spec, int32_t len, int32_t d, DevKernel* k);

__host__ __device__ inline bool is_stationary(int type) {
  return type == GPB_KERNEL_RBF || type == GPB_KERNEL_MATERN12 || type == GPB_KERNEL_MATERN32 ||
         type == GPB_KERNEL_MATERN52 || type == GPB_KERNEL_RQ;
}

// --------------------------------------------------------------------------
// Device evaluation of one leaf for the pair (xi, xj) (raw inputs, length d).
// If `g` is non-null it receives dk/dtheta for the leaf's own parameters
// (indices relative to the leaf's first parameter).
// --------------------------------------------------------------------------
__device__ __forceinline__ float leaf_eval(const DevKernel& K, const LeafDesc& L, const float* xi,
                                           const float* xj, float* g) {
  const float* p = K.params + L.pofs;
  const int nd = L.ndims;
  switch (L.type) {
    case GPB_KERNEL_RBF:
    case GPB_KERNEL_MATERN12:
    case GPB_KERNEL_MATERN32:
    case GPB_KERNEL_MATERN52:
    case GPB_KERNEL_RQ: {
      // s = sum_k (diff_k / l_k)^2
      float s = 0.f;
      if (L.ard) {
        for (int k = 0; k < nd; ++k) {
          const float dk = (xi[L.dims[k]] - xj[L.dims[k]]) / p[k];
          s = fmaf(dk, dk, s);
        }
      } else {
        for (int k = 0; k < nd; ++k) {
          const float dk = xi[L.dims[k]] - xj[L.dims[k]];
          s = fmaf(dk, dk, s);
        }
        s = s / (p[0] * p[0]);
      }
      const int nl = L.ard ? nd : 1;
      float os = 1.f, kval, psi;  // psi = -2 dk/ds
      if (L.type == GPB_KERNEL_RQ) {
        const float alpha = p[nl];
        os = p[nl + 1];
        const float z = s / (2.f * alpha);
        const float base = 1.f + z;
        const float powv = powf(base, -alpha);
        kval = os * powv;
        psi = os * powv / base;
        if (g) g[nl] = kval * (z / base - logf(base));
      } else {
        os = p[nl];
        if (L.type == GPB_KERNEL_RBF) {
          const float e = expf(-0.5f * s);
          kval = os * e;
          psi = kval;
        } else {
          const float r = sqrtf(fmaxf(s + 1e-20f, 1e-20f));
          if (L.type == GPB_KERNEL_MATERN12) {
            const float a = L.ard ? fmaxf(-r, -20.f) : -r;
            const float e = expf(a);
            kval = os * e;
            psi = os * e / r;
          } else if (L.type == GPB_KERNEL_MATERN32) {
            const float r3 = 1.7320508075688772f * r;
            const float e = expf(fmaxf(-r3, -20.f));
            kval = os * (1.f + r3) * e;
            psi = 3.f * os * e;
          } else {
            const float r5 = 2.23606797749979f * r;
            const float e = expf(fmaxf(-r5, -20.f));
            kval = os * (1.f + r5 + (5.f / 3.f) * s) * e;
            psi = (5.f / 3.f) * os * (1.f + r5) * e;
          }
        }
      }
      if (g) {
        g[L.type == GPB_KERNEL_RQ ? nl + 1 : nl] = kval / os;
        if (L.ard) {
          for (int k = 0; k < nd; ++k) {
            const float dk = (xi[L.dims[k]] - xj[L.dims[k]]) / p[k];
            g[k] = psi * dk * dk / p[k];
          }
        } else {
          g[0] = psi * s / p[0];
        }
      }
      return kval;
    }
    case GPB_KERNEL_PERIODIC: {
      const int nl = L.ard ? nd : 1;
      const float period = p[nl];
      const float os = p[nl + 1];
      const float w = 3.14159265358979f / period;
      float arg = 0.f;      // sum_k sin^2_k / l_k
      float dper = 0.f;     // sum_k sin_k cos_k diff_k / l_k
      for (int k = 0; k < nd; ++k) {
        const float diff = xi[L.dims[k]] - xj[L.dims[k]];
        float sn, cs;
        sincosf(w * diff, &sn, &cs);
        const float lk = L.ard ? p[k] : 1.f;
        arg += sn * sn / lk;
        dper += sn * cs * diff / lk;
        if (g && L.ard) g[k] = sn * sn / (lk * lk);  // scaled by 2k below
      }
      if (!L.ard) {
        arg /= p[0];
        dper /= p[0];
      }
      const float e = expf(-2.f * arg);
      const float kval = os * e;
      if (g) {
        if (L.ard) {
          for (int k = 0; k < nd; ++k) g[k] *= 2.f * kval;
        } else {
          g[0] = 2.f * kval * arg / p[0];
        }
        g[nl] = kval * 4.f * 3.14159265358979f / (period * period) * dper;
        g[nl + 1] = e;
      }
      return kval;
    }
    case GPB_KERNEL_LINEAR: {
      const float os = p[L.ard ? nd : 1];
      float dot = 0.f;
      if (L.ard) {
        for (int k = 0; k < nd; ++k) {
          const float prod = xi[L.dims[k]] * xj[L.dims[k]];
          dot = fmaf(p[k], prod, dot);
          if (g) g[k] = os * prod;
        }
        if (g) g[nd] = dot;
        return os * dot;
      }
      for (int k = 0; k < nd; ++k) dot = fmaf(xi[L.dims[k]], xj[L.dims[k]], dot);
      if (g) {
        g[0] = os * dot;
        g[1] = p[0] * dot;
      }
      return os * p[0] * dot;
    }
    case GPB_KERNEL_POLYNOMIAL: {
      // iso: [degree, offset, os]; ARD: [var_0..var_{k-1}, degree, offset, os]
      const int base_i = L.ard ? nd : 0;
      const int degree = (int)lrintf(p[base_i]);
      const float offset = p[base_i + 1];
      const float os = p[base_i + 2];
      float dot = 0.f;
      for (int k = 0; k < nd; ++k) {
        const float prod = xi[L.dims[k]] * xj[L.dims[k]];
        dot = L.ard ? fmaf(p[k], prod, dot) : dot + prod;
      }
      const float base = dot + offset;
      float pw1 = 1.f;  // base^(degree-1)
      for (int q = 1; q < degree; ++q) pw1 *= base;
      const float pw = pw1 * base;
      if (g) {
        const float dbase = os * (float)degree * pw1;
        if (L.ard) {
          for (int k = 0; k < nd; ++k) g[k] = dbase * xi[L.dims[k]] * xj[L.dims[k]];
        }
        g[base_i] = 0.f;  // fixed integer degree: not trainable
        g[base_i + 1] = dbase;
        g[base_i + 2] = pw;
      }
      return os * pw;
    }
  }
  return 0.f;
}

// Full tree value; if `grad` (length nparams) is non-null it receives
// dK/dtheta_p for every parameter via reverse accumulation over the post-order
// program.
template <bool kGrad>
__device__ __forceinline__ float tree_eval(const DevKernel& K, const float* xi, const float* xj,
                                           float* grad) {
  float val[GPB_MAX_NODES];
  int child0[GPB_MAX_NODES], child1[GPB_MAX_NODES];
  int stack[GPB_MAX_NODES];
  int sp = 0;
  for (int nidx = 0; nidx < K.nnodes; ++nidx) {
    const int op = K.node_op[nidx];
    if (op == GPB_NODE_LEAF) {
      val[nidx] = leaf_eval(K, K.leaf[K.node_arg[nidx]], xi, xj, nullptr);
      child0[nidx] = child1[nidx] = -1;
      stack[sp++] = nidx;
    } else if (op == GPB_NODE_SCALE) {
      const int a = stack[--sp];
      val[nidx] = K.params[K.node_arg[nidx]] * val[a];
      child0[nidx] = a;
      child1[nidx] = -1;
      stack[sp++] = nidx;
    } else {
      const int b = stack[--sp];
      const int a = stack[--sp];
      val[nidx] = (op == GPB_NODE_SUM) ? val[a] + val[b] : val[a] * val[b];
      child0[nidx] = a;
      child1[nidx] = b;
      stack[sp++] = nidx;
    }
  }
  const int root = K.nnodes - 1;
  if constexpr (kGrad) {
    float adj[GPB_MAX_NODES];
    for (int nidx = 0; nidx < K.nnodes; ++nidx) adj[nidx] = 0.f;
    adj[root] = 1.f;
    for (int nidx = root; nidx >= 0; --nidx) {
      const int op = K.node_op[nidx];
      const float a_n = adj[nidx];
      if (op == GPB_NODE_LEAF) {
        const LeafDesc& L = K.leaf[K.node_arg[nidx]];
        float g[GPB_MAX_DIM + 3];
        leaf_eval(K, L, xi, xj, g);
        const int np = leaf_num_params(L.type, L.ard, L.ndims);
        for (int q = 0; q < np; ++q) grad[L.pofs + q] = a_n * g[q];
      } else if (op == GPB_NODE_SCALE) {
        adj[child0[nidx]] += a_n * K.params[K.node_arg[nidx]];
        grad[K.node_arg[nidx]] = a_n * val[child0[nidx]];
      } else if (op == GPB_NODE_SUM) {
        adj[child0[nidx]] += a_n;
        adj[child1[nidx]] += a_n;
      } else {
        adj[child0[nidx]] += a_n * val[child1[nidx]];
        adj[child1[nidx]] += a_n * val[child0[nidx]];
      }
    }
  }
  return val[root];
}

}  // namespace gpb
