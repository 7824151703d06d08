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
    t13 = t10[2]
    t14 = mx.fast.scaled_dot_product_attention(t11, t12, t13, scale=0.08838834764831843)
    t15 = mx.transpose(t14, [0, 2, 1, 3])
    t16 = mx.reshape(t15, [t15.shape[0], t15.shape[1], -1])
    t17 = t16 @ x3
    t18 = x0 + t17
    t19 = t18 @ x4
    t20 = t18 * t18
    t21 = mx.mean(t20, axis=[2], keepdims=True)
    c22 = mx.array(1e-05, dtype=mx.bfloat16)
    t23 = t21 + c22
    t24 = mx.rsqrt(t23)
    t25 = t19 * t24
    t26 = mx.sigmoid(t25)
    t27 = t25 * t26
    t28 = t18 @ x5
    t29 = t28 * t24
    t30 = t27 * t29
    t31 = t30 @ x6
    t32 = t18 + t31
    return t32
