"""Measurement helpers of the B200 build: calibration data and the P_ch sweep."""

from .calibration import CalibrationData, calibration_fingerprint, calibration_from_images
from .p_ch import default_p_candidates, measure_p_ch, sweep_p_ch

__all__ = ["CalibrationData", "calibration_fingerprint", "calibration_from_images", "default_p_candidates",
           "measure_p_ch", "sweep_p_ch"]
