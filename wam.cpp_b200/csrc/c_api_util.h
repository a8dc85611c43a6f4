// Helpers shared by the C ABI translation units.
#pragma once

#include <string>

namespace wamb {

void set_last_error(const std::string& msg);
int num_sms_current();
// WAM_B200_OK if the current device is sm_100 (B200), else an error code and a reason.
int check_sm100(std::string* why);

}  // namespace wamb
