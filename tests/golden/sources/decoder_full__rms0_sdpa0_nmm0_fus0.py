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
    t9 = mx.reshape(t8, [t8.shape[0], t8.shape[1], 3, 32, 128])
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
    t25 = t24 @ x4
    t26 = t24 * t24
    t27 = mx.mean(t26, axis=[2], keepdims=True)
    c28 = mx.array(1e-05, dtype=mx.bfloat16)
    t29 = t27 + c28
    t30 = mx.rsqrt(t29)
    t31 = t25 * t30
    t32 = mx.sigmoid(t31)
    t33 = t31 * t32
    t34 = t24 @ x5
    t35 = t34 * t30
    t36 = t33 * t35
    t37 = t36 @ x6
    t38 = t24 + t37
    return t38
