"""Progressive MoE layer: configs, inputs, the B200 data plane, the oracle and the checker."""

from .config import CASE_ORDER, CASE_SPECS, MoELayerConfig, PRESETS, load_config, preset, r4_case

__all__ = ["CASE_ORDER", "CASE_SPECS", "MoELayerConfig", "PRESETS", "load_config", "preset", "r4_case"]


def __getattr__(name):
    if name == "ProgressiveMoELayer":
        from .layer import ProgressiveMoELayer

        return ProgressiveMoELayer
    raise AttributeError(name)
