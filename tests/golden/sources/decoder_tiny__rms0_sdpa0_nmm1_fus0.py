import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, x2, x3, x4, x5, x6, x7, *_, **__):
    t1 = x0 * x0
    t2 = mx.mean(t1, axis=[2], keepdims=True)
    c3 = mx.array(1e-05, dtype=mx.bfloat16)
    t4 = t2 + c3
    t5 = mx.rsqrt(t4)
    t6 = x0 * t5
    t7 = t6 * x1
    t8 = t7 @ x2
    t9 = mx.reshape(t8, [t8.shape[0], t8.shape[1], 3, 2, 128])
    t10 = mx.transpose(t9, [2, 0, 3, 1, 4])
    t11 = t10[0]
    t12 = t10[1]
    t13 = mx.transpose(t12, [0, 1, 3, 2])
    t14 = t11 @ t13
    c15 = mx.array(0.08838834764831843, dtype=mx.bfloat16)
    t16 = t14 * c15
    t17 = t16 + x7
    t18 = mx.softmax(t17, axis=3)
    t19 = t10[2]
    t20 = t18 @ t19
    t21 = mx.transpose(t20, [0, 2, 1, 3])
    t22 = mx.reshape(t21, [t21.shape[0], t21.shape[1], -1])
    t23 = t22 @ x3
    t24 = x0 + t23
    t25 = mx.fast.rms_norm(t24, None, eps=1e-05)
    t26 = t25 @ x4
    t27 = mx.sigmoid(t26)
    t28 = t26 * t27
    t29 = mx.fast.rms_norm(t24, None, eps=1e-05)
    t30 = t29 @ x5
    t31 = t28 * t30
    t32 = t31 @ x6
    t33 = t24 + t32
    return t33
