// fuse_chains.chain
module {
  func.func @fuse_chains__chain(%arg0: tensor<8x16xf32>, %arg1: tensor<8x16xf32>) -> tensor<8x16xf32> {
    %0 = fp.add %arg0, %arg1 : tensor<8x16xf32>
    %1 = fp.scale %0 {factor = 2.000000000e+00 : f32} : tensor<8x16xf32>
    %2 = fp.relu %1 : tensor<8x16xf32>
    %3 = fp.exp %2 : tensor<8x16xf32>
    return %3 : tensor<8x16xf32>
  }
}

// fuse_chains.multiuse
module {
  func.func @fuse_chains__multiuse(%arg0: tensor<4x4xf32>) -> (tensor<4x4xf32>, tensor<4x4xf32>) {
    %0 = fp.relu %arg0 : tensor<4x4xf32>
    %1 = fp.exp %0 : tensor<4x4xf32>
    %2 = fp.scale %0 {factor = 3.000000000e+00 : f32} : tensor<4x4xf32>
    return %1, %2 : tensor<4x4xf32>, tensor<4x4xf32>
  }
}

// fuse_chains.softmax_chain
module {
  func.func @fuse_chains__softmax_chain(%arg0: tensor<4x64xf32>) -> tensor<4x64xf32> {
    %0 = fp.scale %arg0 {factor = 5.000000000e-01 : f32} : tensor<4x64xf32>
    %1 = fp.softmax %0 {axis = 1 : i64} : tensor<4x64xf32>
    %2 = fp.relu %1 : tensor<4x64xf32>
    return %2 : tensor<4x64xf32>
  }
}

// fuse_chains.softmax_axis0
module {
  func.func @fuse_chains__softmax_axis0(%arg0: tensor<4x64xf32>) -> tensor<4x64xf32> {
    %0 = fp.scale %arg0 {factor = 5.000000000e-01 : f32} : tensor<4x64xf32>
    %1 = fp.softmax %0 {axis = 0 : i64} : tensor<4x64xf32>
    return %1 : tensor<4x64xf32>
  }
}

// fuse_chains.dedupe
module {
  func.func @fuse_chains__dedupe(%arg0: tensor<4x4xf32>) -> tensor<4x4xf32> {
    %0 = fp.mul %arg0, %arg0 : tensor<4x4xf32>
    %1 = fp.relu %0 : tensor<4x4xf32>
    return %1 : tensor<4x4xf32>
  }
}

// fuse_attention.attn
module {
  func.func @fuse_attention__attn(%arg0: tensor<2x4x32x64xf16>, %arg1: tensor<2x4x32x64xf16>, %arg2: tensor<2x4x32x64xf16>) -> tensor<2x4x32x64xf16> {
    %0 = fp.transpose %arg1 : tensor<2x4x32x64xf16> -> tensor<2x4x64x32xf16>
    %1 = fp.matmul %arg0, %0 : (tensor<2x4x32x64xf16>, tensor<2x4x64x32xf16>) -> tensor<2x4x32x32xf16>
    %2 = fp.scale %1 {factor = 5.000000000e-01 : f32} : tensor<2x4x32x32xf16>
    %3 = fp.scale %2 {factor = 5.000000000e-01 : f32} : tensor<2x4x32x32xf16>
    %4 = fp.softmax %3 {axis = 3 : i64} : tensor<2x4x32x32xf16>
    %5 = fp.matmul %4, %arg2 : (tensor<2x4x32x32xf16>, tensor<2x4x32x64xf16>) -> tensor<2x4x32x64xf16>
    return %5 : tensor<2x4x32x64xf16>
  }
}

// fuse_attention.attn_multiuse
module {
  func.func @fuse_attention__attn_multiuse(%arg0: tensor<1x2x16x16xf32>, %arg1: tensor<1x2x16x16xf32>, %arg2: tensor<1x2x16x16xf32>) -> (tensor<1x2x16x16xf32>, tensor<1x2x16x16xf32>) {
    %0 = fp.transpose %arg1 : tensor<1x2x16x16xf32> -> tensor<1x2x16x16xf32>
    %1 = fp.matmul %arg0, %0 : (tensor<1x2x16x16xf32>, tensor<1x2x16x16xf32>) -> tensor<1x2x16x16xf32>
    %2 = fp.softmax %1 {axis = 3 : i64} : tensor<1x2x16x16xf32>
    %3 = fp.matmul %2, %arg2 : (tensor<1x2x16x16xf32>, tensor<1x2x16x16xf32>) -> tensor<1x2x16x16xf32>
    return %3, %2 : tensor<1x2x16x16xf32>, tensor<1x2x16x16xf32>
  }
}

// dedupe_mul.dedupe
module {
  func.func @dedupe_mul__dedupe(%arg0: tensor<4x4xf32>) -> tensor<4x4xf32> {
    %0 = fp.mul %arg0, %arg0 : tensor<4x4xf32>
    %1 = fp.relu %0 : tensor<4x4xf32>
    return %1 : tensor<4x4xf32>
  }
}

// two_softmax.two_sm
module {
  func.func @two_softmax__two_sm(%arg0: tensor<4x8xf32>) -> tensor<4x8xf32> {
    %0 = fp.softmax %arg0 {axis = 1 : i64} : tensor<4x8xf32>
    %1 = fp.softmax %0 {axis = 1 : i64} : tensor<4x8xf32>
    return %1 : tensor<4x8xf32>
  }
}

// no_fuse_head_dim.attn_d24
module {
  func.func @no_fuse_head_dim__attn_d24(%arg0: tensor<1x2x8x24xf32>, %arg1: tensor<1x2x8x24xf32>, %arg2: tensor<1x2x8x24xf32>) -> tensor<1x2x8x24xf32> {
    %0 = fp.transpose %arg1 : tensor<1x2x8x24xf32> -> tensor<1x2x24x8xf32>
    %1 = fp.matmul %arg0, %0 : (tensor<1x2x8x24xf32>, tensor<1x2x24x8xf32>) -> tensor<1x2x8x8xf32>
    %2 = fp.scale %1 {factor = 2.500000000e-01 : f32} : tensor<1x2x8x8xf32>
    %3 = fp.softmax %2 {axis = 3 : i64} : tensor<1x2x8x8xf32>
    %4 = fp.matmul %3, %arg2 : (tensor<1x2x8x8xf32>, tensor<1x2x8x24xf32>) -> tensor<1x2x8x24xf32>
    return %4 : tensor<1x2x8x24xf32>
  }
}
