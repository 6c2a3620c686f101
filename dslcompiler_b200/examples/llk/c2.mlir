func.func @mm(%a: tensor<4096x4096xbf16>, %b: tensor<4096x4096xbf16>, %c: tensor<4096x4096xf32>) -> tensor<4096x4096xf32> {
  %0 = llk.matmul ins(%a, %b : tensor<4096x4096xbf16>, tensor<4096x4096xbf16>)
      outs(%c : tensor<4096x4096xf32>) {accumulator_type = f32, math_mode = #llk.math_mode<strict>}
      -> tensor<4096x4096xf32>
  return %0 : tensor<4096x4096xf32>
}
