// Test infrastructure: a minimal stand-in for pytoast's <toast/math/scalar.h>
// (see toast/utils/vector_math.h in this tree for why): the scalar-type tag
// the reference passes to normalize_bwd<Float32>.
#pragma once

struct Float32 {};
