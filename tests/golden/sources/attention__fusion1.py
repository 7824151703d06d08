import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, x2, x3, *_, **__):
    t1 = mx.fast.scaled_dot_product_attention(x0, x1, x2, scale=0.08838834764831843)
    return t1
