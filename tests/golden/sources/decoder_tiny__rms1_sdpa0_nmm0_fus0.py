import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, x2, x3, x4, x5, x6, x7, *_, **__):
    t1 = mx.fast.rms_norm(x0, x1, eps=1e-05)
    t2 = t1 @ x2
    t3 = mx.reshape(t2, [t2.shape[0], t2.shape[1], 3, 2, 128])
    t4 = mx.transpose(t3, [2, 0, 3, 1, 4])
    t5 = t4[0]
    t6 = t4[1]
    t7 = mx.transpose(t6, [0, 1, 3, 2])
    t8 = t5 @ t7
    c9 = mx.array(0.08838834764831843, dtype=mx.bfloat16)
    t10 = t8 * c9
    t11 = t10 + x7
    t12 = mx.softmax(t11, axis=3)
    t13 = t4[2]
    t14 = t12 @ t13
    t15 = mx.transpose(t14, [0, 2, 1, 3])
    t16 = mx.reshape(t15, [t15.shape[0], t15.shape[1], -1])
    t17 = t16 @ x3
    t18 = x0 + t17
    t19 = t18 @ x5
    t20 = t18 @ x4
    t21 = t18 * t18
    t22 = mx.mean(t21, axis=[2], keepdims=True)
    c23 = mx.array(1e-05, dtype=mx.bfloat16)
    t24 = t22 + c23
    t25 = mx.rsqrt(t24)
    t26 = t20 * t25
    t27 = mx.sigmoid(t26)
    t28 = mx.fast.rms_norm(t20, t27, eps=1e-05)
    t29 = mx.fast.rms_norm(t19, t28, eps=1e-05)
    t30 = t29 @ x6
    t31 = t18 + t30
    return t31
