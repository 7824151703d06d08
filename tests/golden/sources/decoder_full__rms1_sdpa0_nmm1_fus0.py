import phew_b200.mx as mx
from phew_b200.mx import fast

@mx.compile
def optimized(x0, x1, x2, x3, x4, x5, x6, x7, *_, **__):
    t1 = mx.fast.rms_norm(x0, x1, eps=1e-05)
    t2 = t1 @ x2
    t3 = mx.reshape(t2, [t2.shape[0], t2.shape[1], 3, 32, 128])
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
    t21 = mx.fast.rms_norm(t18, None, eps=1e-05)
    t22 = t21 @ x4
    t23 = mx.sigmoid(t22)
    t24 = mx.fast.rms_norm(t20, t23, eps=1e-05)
    t25 = mx.fast.rms_norm(t19, t24, eps=1e-05)
    t26 = t25 @ x6
    t27 = t18 + t26
    return t27
