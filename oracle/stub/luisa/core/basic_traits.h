// Test-infrastructure stub: lets the reference's CPU codec header compile
// without LuisaCompute. Only the two names that header needs are provided.
#pragma once
namespace luisa {
using half = _Float16;
}
#define LUISA_STRUCT(S, ...) struct S##_lcml_oracle_stub
