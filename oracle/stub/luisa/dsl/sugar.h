// Test-infrastructure stub (empty): the CPU half of the codec needs no DSL.
#pragma once
