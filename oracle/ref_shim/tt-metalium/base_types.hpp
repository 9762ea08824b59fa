// TEST INFRASTRUCTURE: empty stand-in (see host_api.hpp).
#pragma once
