// slx_status.h -- status codes shared by the host sources (the public definitions live in slx.h).
#pragma once
#include "slx.h"
