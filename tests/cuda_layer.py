"""Factories for the CUDA layers used by the -m gpu tests."""
import sili__new_b200 as S


def cuda_det(n_in, n_out, mw):
    return S.SparseLinearLayerDeterministic(n_in, n_out, mw)


def cuda_stoch(n_in, n_out, mw):
    return S.SparseLinearLayer(n_in, n_out, mw)
