import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x, w, *_, **__):
    t1 = mx.fast.rms_norm(x, w, eps=1e-05)
    return t1
