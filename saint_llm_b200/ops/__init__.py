"""Operator layer: eager references and the sm_100a native kernels behind one API."""
