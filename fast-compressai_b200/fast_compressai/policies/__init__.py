"""Selection policies of the B200 build (P_ch of the warp_div coder)."""

from .p_ch import PChSelection, choose_p_ch, legal_p_candidates

__all__ = ["PChSelection", "choose_p_ch", "legal_p_candidates"]
