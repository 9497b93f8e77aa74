"""matrix_numbers_b200 -- B200-native (sm_100a) FP64 GEMM from INT8 residue planes and CRT reconstruction.

A from-scratch rebuild of the FP64-on-INT8 engine of dl1683/matrix-numbers (code/ozaki_engine.py) behind the same
Python entry point:

    from matrix_numbers_b200 import OzakiCRT
    C, info = OzakiCRT().run(A, B)            # A (m, k), B (k, n): float64 CUDA tensors

The package directory is named ``matrix-numbers_b200``; ``__graft_entry__.load_package()`` (repository root)
registers it under the importable name ``matrix_numbers_b200``.  The compute path is libozaki_b200.so (hand-written
sm_100a kernels behind the C ABI in include/ozaki_b200.h); there is no CPU path.
"""
from . import _lib
from .constants import (MODS, NEG, NMAX, _limbs_for, _pow2tab, bound_matrix, limbs_for, make_config_table,
                        modulus_product, pick_config, pmax_bits, sigma_of, worst_case_p)


def __getattr__(name):
    # torch-dependent modules are imported lazily so that the host helpers work without initialising CUDA
    if name in ("OzakiCRT", "DEV"):
        from . import engine
        return getattr(engine, name)
    if name in ("DistributedOzakiCRT",):
        from . import distributed
        return getattr(distributed, name)
    if name in ("PersistA",):
        from . import persist
        return getattr(persist, name)
    if name in ("full_certificate",):
        from . import certificate
        return getattr(certificate, name)
    if name in ("ResidueChain", "planes_for", "chain_bound"):
        from . import chain
        return getattr(chain, name)
    if name in ("coprime_ip", "int8_crt", "chain_cost_model"):
        from . import planning
        return getattr(planning, name)
    if name in ("make_inputs", "make_inputs_w", "config_inputs", "Sample", "exact_sample", "audit_bound", "CONFIGS",
                "AccuracySample", "correctly_rounded_products", "two_products"):
        from . import measure
        return getattr(measure, name)
    raise AttributeError(name)


__all__ = ["OzakiCRT", "DistributedOzakiCRT", "PersistA", "full_certificate", "MODS", "NMAX", "NEG", "pmax_bits", "bound_matrix", "worst_case_p",
           "sigma_of", "make_config_table", "pick_config", "limbs_for", "_limbs_for", "_pow2tab", "modulus_product",
           "make_inputs", "make_inputs_w", "config_inputs", "Sample", "exact_sample", "audit_bound", "CONFIGS",
           "AccuracySample", "correctly_rounded_products", "two_products", "coprime_ip", "int8_crt",
           "chain_cost_model", "ResidueChain", "planes_for", "chain_bound", "_lib"]
