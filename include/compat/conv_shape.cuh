// conv_shape.cuh - drop-in shim under the reference's header name.
//
// Code written against pthodima/int8_kernel_lab includes include/conv_shape.cuh;
// with include/compat on the include path ahead of the reference's headers,
// the same #include pulls in this engine's ConvShape, launchers and
// eligibility predicate (include/int8conv.hpp) instead.  Link libint8conv.so.
#pragma once
#include "int8conv.hpp"
