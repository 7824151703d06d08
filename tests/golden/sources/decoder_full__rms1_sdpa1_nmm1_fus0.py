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
    t7 = t4[2]
    t8 = mx.fast.scaled_dot_product_attention(t5, t6, t7, scale=0.08838834764831843)
    t9 = mx.transpose(t8, [0, 2, 1, 3])
    t10 = mx.reshape(t9, [t9.shape[0], t9.shape[1], -1])
    t11 = t10 @ x3
    t12 = x0 + t11
    t13 = t12 @ x5
    t14 = t12 @ x4
    t15 = mx.fast.rms_norm(t12, None, eps=1e-05)
    t16 = t15 @ x4
    t17 = mx.sigmoid(t16)
    t18 = mx.fast.rms_norm(t14, t17, eps=1e-05)
    t19 = mx.fast.rms_norm(t13, t18, eps=1e-05)
    t20 = t19 @ x6
    t21 = t12 + t20
    return t21
