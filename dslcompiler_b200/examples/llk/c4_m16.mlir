func.func @f(%x: tensor<16x4096xbf16>, %wg: tensor<4096x14336xbf16>, %wu: tensor<4096x14336xbf16>, %init: tensor<16x14336xbf16>) -> tensor<16x14336xbf16> {
  %y = llk.fused_swiglu ins(%x, %wg, %wu : tensor<16x4096xbf16>, tensor<4096x14336xbf16>, tensor<4096x14336xbf16>)
      outs(%init : tensor<16x14336xbf16>)
      {accumulator_type = f32, activation = #llk.activation<silu>, math_mode = #llk.math_mode<strict>}
      -> tensor<16x14336xbf16>
  return %y : tensor<16x14336xbf16>
}
