func.func @f(%x: tensor<2048x4096xbf16>, %wg: tensor<4096x11008xbf16>, %wu: tensor<4096x11008xbf16>, %init: tensor<2048x11008xbf16>) -> tensor<2048x11008xbf16> {
  %y = llk.fused_swiglu ins(%x, %wg, %wu : tensor<2048x4096xbf16>, tensor<4096x11008xbf16>, tensor<4096x11008xbf16>)
      outs(%init : tensor<2048x11008xbf16>)
      {accumulator_type = f32, activation = #llk.activation<silu>, math_mode = #llk.math_mode<strict>}
      -> tensor<2048x11008xbf16>
  return %y : tensor<2048x11008xbf16>
}
