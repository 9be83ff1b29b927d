"""ctypes mirrors of the C structs in ``include/bifrost_b200.h``."""
import ctypes

_P = ctypes.c_void_p


class BfLayer(ctypes.Structure):
    _fields_ = [("wbuf", _P), ("ab_b", _P), ("mix_b", _P), ("mix_lse", _P), ("mem_scale", _P), ("A_log", _P),
                ("dt_bias", _P), ("decay_mask", _P), ("H", ctypes.c_int), ("G", ctypes.c_int),
                ("D", ctypes.c_int), ("d", ctypes.c_int), ("window", ctypes.c_int), ("sinks", ctypes.c_int)]


class BfRingCache(ctypes.Structure):
    _fields_ = [("ring_k", _P), ("ring_v", _P), ("ring_km", _P), ("ring_g", _P), ("ring_beta", _P),
                ("ring_pos", _P), ("ring_pos_bstride", ctypes.c_longlong), ("sink_k", _P), ("sink_v", _P),
                ("ns", ctypes.c_int), ("S", _P)]
