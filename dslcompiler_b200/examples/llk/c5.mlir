func.func @f(%x: tensor<8192x8192xbf16>, %wg: tensor<8192x28672xbf16>, %wu: tensor<8192x28672xbf16>, %init: tensor<8192x28672xbf16>) -> tensor<8192x28672xbf16> {
  %y = llk.fused_swiglu ins(%x, %wg, %wu : tensor<8192x8192xbf16>, tensor<8192x28672xbf16>, tensor<8192x28672xbf16>)
      outs(%init : tensor<8192x28672xbf16>)
      {accumulator_type = f32, activation = #llk.activation<silu>, math_mode = #llk.math_mode<strict>}
      -> tensor<8192x28672xbf16>
  return %y : tensor<8192x28672xbf16>
}
