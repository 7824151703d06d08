import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, x2, x3, *_, **__):
    t1 = x0 * x1
    t2 = t1 + x2
    c3 = mx.array(0.5, dtype=mx.float16)
    t4 = t2 * c3
    t5 = t2 * t2
    t6 = t5 * t2
    c7 = mx.array(0.044715, dtype=mx.float16)
    t8 = t6 * c7
    t9 = t2 + t8
    c10 = mx.array(0.7978845608028654, dtype=mx.float16)
    t11 = t9 * c10
    t12 = mx.tanh(t11)
    c13 = mx.array(1.0, dtype=mx.float16)
    t14 = t12 + c13
    t15 = t4 * t14
    t16 = mx.sigmoid(x3)
    t17 = t15 * t16
    t18 = t17 + x0
    return t18
