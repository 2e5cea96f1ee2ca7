"""Locations of the in-tree native libraries."""
import os

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
BACKEND_LIB = os.path.join(PKG, "libhymt2_cuda.so")
# the same backend with the per-phase %globaltimer timeline compiled in
# (-DHYK_TRACE); built only on request, for measurements
TRACE_LIB = os.path.join(PKG, "libhymt2_cuda_trace.so")
BACKEND_ARCHIVE = os.path.join(PKG, "libhymt2_cuda.a")
SYNTH_LIB = os.path.join(PKG, "libhysynth.so")
