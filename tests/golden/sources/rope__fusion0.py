import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, *_, **__):
    t1 = mx.fast.rope(x0, 128, traditional=False, base=10000.0, scale=1.0, offset=0)
    return t1
