"""Locations of the in-tree native libraries."""
import os

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
BACKEND_LIB = os.path.join(PKG, "libhymt2_cuda.so")
BACKEND_ARCHIVE = os.path.join(PKG, "libhymt2_cuda.a")
SYNTH_LIB = os.path.join(PKG, "libhysynth.so")
